"""Host-driven token step for the two paths the device engines do not plan:
flashnano-1.6 (chunk relays) and FlashLighting 2.0 with memory slots (latent
attention with weighted compaction).  Neither is a BASELINE configuration;
FlashLighting without memory slots runs on the decode kernel and Heavy Medium
on its device token step (csrc/heavy.cu).

One token runs the way the reference's ``MiracleModel._step`` does
(miracle_reasoning/model.py:95-190, 257-285): the host sequences the op
kernels (csrc/ops.cu, each the reference's kernels.cl work item restated in
CUDA) and makes the latent compaction decision with the same float32 NumPy
expressions.  What changes is where the weights live: they stay resident in
HBM in their stored dtype, and every projection reads them there
(``mr_model_linear``, bit-identical to the reference's linear over widened
weights).  The op kernels reproduce the reference's per-element arithmetic, so
logits and decisions follow the reference's.

Each step records its discrete decisions in ``decisions`` (one dict per layer:
``latent_positions``, ``memory_size``), which the parity tests compare with
the reference's.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native
from .weights import expected_shapes

FAMILIES = ("flashnano-1.6", "flashlighting-2.0")


class Ring:
    """KV ring (model.py:15-33): entry i at (count % capacity) * width."""

    def __init__(self, backend, capacity, width):
        self.k = backend.empty((capacity, width))
        self.v = backend.empty((capacity, width))
        self.count, self.capacity, self.width = 0, capacity, width

    def append(self, backend, key, value):
        slot = (self.count % self.capacity) * self.width
        backend.copy(key, self.k, target_offset=slot)
        backend.copy(value, self.v, target_offset=slot)
        self.count += 1

    @property
    def length(self):
        return min(self.count, self.capacity)

    @property
    def start(self):
        return (self.count - self.length) % self.capacity


class OpStepper:
    """One sequence of a flashnano-1.6 model or of a FlashLighting model with memory slots."""

    def __init__(self, model):
        self.model, self.config, self.b = model, model.config, model.backend
        self.context_length = model.context_length
        self.shapes = expected_shapes(self.config)
        self.frequencies = self.b.upload(np.ascontiguousarray(self.config.inverse_frequencies(), dtype=np.float32))
        self._device, self._host = {}, {}
        self.reset()

    def reset(self):
        self.position = 0
        self.states = [{} for _ in range(self.config.layers)]
        self.decisions = []

    # resident tensors ------------------------------------------------------------
    def tensor(self, name):
        """Float32 device copy of a small tensor (norm gains, relay queries), kept."""
        t = self._device.get(name)
        if t is None:
            shape = self.shapes[name]
            t = self.b.empty(shape)
            rows = shape[0] if len(shape) == 2 else 1
            _native.call("mr_model_tensor_rows", self.model._handle, name.encode(), 0, rows, t.handle)
            self._device[name] = t
        return t

    def host(self, name):
        """Float32 host copy of a small tensor (gates, router biases), kept."""
        a = self._host.get(name)
        if a is None:
            a = np.empty(self.shapes[name], dtype=np.float32)
            _native.call("mr_model_tensor_download", self.model._handle, name.encode(),
                         a.ctypes.data_as(C.POINTER(C.c_float)), a.size)
            self._host[name] = a
        return a

    def linear(self, x, name):
        """x[rows, in] . W^T against the resident tensor (model.py:84-85)."""
        rows = x.shape[0]
        out = self.b.empty((rows, self.shapes[name][0]))
        _native.call("mr_model_linear", self.model._handle, name.encode(), x.handle, rows, out.handle)
        return out

    def embed_row(self, token):
        out = self.b.empty((1, self.config.hidden_size))
        _native.call("mr_model_tensor_rows", self.model._handle, b"embed", token, 1, out.handle)
        return out

    # building blocks (model.py:79-93) ---------------------------------------------
    def norm(self, x, name, width=None, eps=None):
        c = self.config
        return self.b.norm(x, self.tensor(name) if name else None, width or c.hidden_size,
                           c.norm_eps if eps is None else eps)

    def ffn(self, x, root):
        return self.linear(self.b.swiglu(self.linear(x, root + "gate"), self.linear(x, root + "up")), root + "down")

    def rotate(self, x, positions, heads):
        return self.b.rotate(x, self.frequencies, positions, heads, self.config.head_dim, self.config.split_half_rope)

    def _note(self, key, value):
        self._layer.setdefault(key, []).append(value)

    # flashnano-1.6: grouped-query attention plus chunk relays (model.py:95-144) -----
    def gqa(self, x, prefix, state, layer, position):
        b, c = self.b, self.config
        kv_heads = c.layer_kv_heads(layer)
        query, key, value = self.linear(x, prefix + "q"), self.linear(x, prefix + "k"), self.linear(x, prefix + "v")
        if c.qk_norm:
            query = self.norm(query, prefix + "q_norm", c.head_dim)
            key = self.norm(key, prefix + "k_norm", c.head_dim)
        query, key = self.rotate(query, position, c.query_heads), self.rotate(key, position, kv_heads)
        ring = state.get("ring")
        if ring is None:
            capacity = min(c.layer_window(layer) or self.context_length, self.context_length)
            ring = state["ring"] = Ring(b, capacity, kv_heads * c.head_dim)
        ring.append(b, key, value)
        relay = state.get("relay")
        attended = b.attention(query, ring.k, ring.v, heads=c.query_heads, kv_heads=kv_heads, dim=c.head_dim,
                               start=ring.start, length=ring.length,
                               extra_keys=relay.k if relay else None, extra_values=relay.v if relay else None,
                               extra_length=relay.count if relay else 0)
        if c.family == "flashnano-1.6":
            self.update_relays(x, prefix, state, kv_heads)
        return self.linear(attended, prefix + "o")

    def update_relays(self, x, prefix, state, kv_heads):
        """Every cbr_chunk_size tokens, pool the chunk into cbr_slots relay keys/values."""
        b, c = self.b, self.config
        chunk, slots, h = c.cbr_chunk_size, c.cbr_slots, c.hidden_size
        if "pending" not in state:
            state["pending"] = b.empty((min(chunk, self.context_length), h))
        offset = self.position % chunk
        b.copy(x, state["pending"], target_offset=offset * h)
        if offset + 1 != chunk:
            return
        queries = b.norm(self.tensor(prefix + "cbr"), None, h, c.cbr_norm_eps)
        scores = b.empty((slots, chunk))
        b.run("pool_scores", (chunk, slots), state["pending"], queries, scores, chunk, slots, h)
        probs = b.softmax(scores)
        pooled, anchors = b.empty((slots, h)), b.empty((slots,))
        b.run("pool_mix", (h, slots), state["pending"], probs, pooled, anchors, chunk, slots, h,
              self.position + 1 - chunk)
        key, value = self.linear(pooled, prefix + "k"), self.linear(pooled, prefix + "v")
        key = self.rotate(self.norm(key, prefix + "k_norm", c.head_dim), anchors, kv_heads)
        relay = state.get("relay")
        width = kv_heads * c.head_dim
        if relay is None:
            relay = state["relay"] = Ring(b, (self.context_length // chunk) * slots, width)
        b.copy(key, relay.k, target_offset=relay.count * width, count=slots * width)
        b.copy(value, relay.v, target_offset=relay.count * width, count=slots * width)
        relay.count += slots

    # FlashLighting latent attention (model.py:146-190) ------------------------------
    def lighting(self, x, prefix, state, position):
        b, c = self.b, self.config
        query = self.rotate(self.norm(self.linear(x, prefix + "q"), prefix + "q_norm", c.head_dim), position,
                            c.query_heads)
        latent = self.norm(self.linear(x, prefix + "latent"), prefix + "latent_norm", c.latent_dim)
        old = state.get("latent")
        n = 0 if old is None else old.shape[0]
        latents = b.empty((n + 1, c.latent_dim))
        if old is not None:
            b.copy(old, latents)
        b.copy(latent, latents, target_offset=n * c.latent_dim)
        positions = state.get("positions", []) + [self.position]
        counts = state.get("counts", []) + [1.0]
        key = self.norm(self.linear(latents, prefix + "k"), prefix + "k_norm", c.head_dim)
        key_positions = b.upload(np.asarray(positions, dtype=np.float32))
        key = self.rotate(key, key_positions, c.kv_heads)
        value = self.linear(latents, prefix + "v")
        scores = b.empty((c.query_heads, n + 1))
        b.run("scores", (n + 1, c.query_heads), query, key, key, scores, c.query_heads, c.kv_heads, c.head_dim,
              n + 1, 0, n + 1, 0)
        b.run("latent_mask", (n + 1, c.query_heads), scores, key_positions, c.query_heads, n + 1,
              state.get("memory_size", 0), self.position - c.window + 1)
        attended = b.mix(b.softmax(scores), value, c.query_heads, c.kv_heads, c.head_dim, 0, n + 1)
        overflow = max(0, n + 1 - c.window)
        if c.memory_slots == 0 and overflow:
            # drop the oldest rows
            kept = b.empty((n + 1 - overflow, c.latent_dim))
            b.copy(latents, kept, source_offset=overflow * c.latent_dim)
            latents, positions, counts, memory_size = kept, positions[overflow:], counts[overflow:], 0
        elif overflow > c.memory_slots:
            # merge rows 0 and 1, weighted by how many tokens each already stands for
            merged = b.empty((n, c.latent_dim))
            a, z = np.float32(counts[0]), np.float32(counts[1])
            b.run("merge_rows", (c.latent_dim,), latents, merged, c.latent_dim, float(a), float(z))
            b.copy(latents, merged, source_offset=2 * c.latent_dim, target_offset=c.latent_dim,
                   count=(n - 1) * c.latent_dim)
            mean = np.float32(np.float32(positions[0]) * a + np.float32(positions[1]) * z) / np.float32(a + z)
            positions = [int(np.rint(mean))] + positions[2:]
            counts = [float(a + z)] + counts[2:]
            latents, memory_size = merged, c.memory_slots
        else:
            memory_size = overflow
        state.update(latent=latents, positions=positions, counts=counts, memory_size=memory_size)
        self._note("latent_positions", list(positions))
        self._note("memory_size", memory_size)
        return self.linear(attended, prefix + "o")

    # one token (model.py:257-285) -------------------------------------------------------
    def step(self, token):
        """Run one token; returns the final-normed hidden state [1, hidden] on the device."""
        b, c = self.b, self.config
        hidden = self.embed_row(int(token))
        position = b.upload(np.asarray([self.position], dtype=np.float32))
        record = []
        for layer, state in enumerate(self.states):
            prefix = f"layers.{layer}."
            self._layer = {}
            if c.family == "flashlighting-2.0":
                normalized = self.norm(hidden, prefix + "a_norm")
                attended = self.lighting(normalized, prefix, state, position)
                attention_gate = float(self.host(prefix + "attention_gate")[0])
                ffn_gate = float(self.host(prefix + "ffn_gate")[0])
                residual = b.add(b.upload(np.zeros(hidden.shape, dtype=np.float32)), attended, attention_gate)
                residual = b.add(residual, self.ffn(normalized, prefix + "ffn."), ffn_gate)
                hidden = b.add(hidden, residual, c.residual_scale)
            else:
                attended = self.gqa(self.norm(hidden, prefix + "a_norm"), prefix, state, layer, position)
                hidden = b.add(hidden, attended, c.residual_scale)
                hidden = b.add(hidden, self.ffn(self.norm(hidden, prefix + "f_norm"), prefix + "ffn."),
                               c.residual_scale)
            record.append(self._layer)
        self.decisions.append(record)
        self.position += 1
        return self.norm(hidden, "norm")

    def logits(self, hidden):
        """Head projection of a step's output, read to the host ([vocab] float32)."""
        head = "embed" if self.config.tie_embeddings else "output"
        return self.b.read(self.linear(hidden, head))[0]
