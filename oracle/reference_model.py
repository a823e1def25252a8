"""CPU oracle of the MiracleReasoning token loop (TEST INFRASTRUCTURE ONLY).

A restatement of the reference's ``MiracleModel`` control flow
(miracle_reasoning/model.py) and ``WeightCache`` (miracle_reasoning/weights.py:
258-297), driving a ``HostBackend`` whose kernels are either the C restatement
(oracle/kernels.c) or the reference's own kernels.cl compiled on the host.
All host-side control arithmetic (heavy block top-k, MoE routing, sampling,
latent-cache compaction) is written with the same float32 NumPy expressions as
the reference, so for the same kernels the results are bit-identical; the
golden fixtures under tests/golden (made by running the reference itself) pin
that.

Besides logits, the oracle records the discrete decisions the parity tests
compare bit for bit: per layer and inner loop the heavy top-k block set, the
MoE expert list and weights, and the latent-cache positions.

Nothing in the product package imports this module; it is the checker.
"""
from __future__ import annotations

import importlib
import math
import sys
from collections import OrderedDict
from pathlib import Path

import numpy as np

_REPO = Path(__file__).resolve().parents[1]
if str(_REPO) not in sys.path:
    sys.path.insert(0, str(_REPO))
_pkg = importlib.import_module("miraclereasoning-cpu_b200")
ModelConfig = _pkg.config.ModelConfig
adapt_weights = _pkg.weights.adapt_weights


class Ring:
    """KV ring (model.py:15-33): offset = (count % capacity) * width."""

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


class WeightCache:
    """Budgeted LRU of widened float32 device weights (weights.py:258-297)."""

    def __init__(self, backend, weights, budget_bytes):
        if type(budget_bytes) is not int or budget_bytes < 4096:
            raise ValueError("weight_cache_bytes must be an integer >= 4096")
        self.backend, self.weights, self.budget = backend, weights, budget_bytes
        self.cache, self.used = OrderedDict(), 0

    def tensor(self, name, start=None, stop=None):
        key = (name, start, stop)
        hit = self.cache.get(key)
        if hit is not None:
            self.cache.move_to_end(key)
            return hit
        raw = self.weights[name]
        array = np.ascontiguousarray(raw if start is None else raw[start:stop], dtype=np.float32)
        while self.cache and self.used + array.nbytes > self.budget:
            _, evicted = self.cache.popitem(last=False)
            self.used -= evicted.size * 4
        tensor = self.backend.upload(array)
        if array.nbytes <= self.budget:
            self.cache[key] = tensor
            self.used += array.nbytes
        return tensor

    def linear(self, x, name):
        rows, inner = self.weights[name].shape
        limit = min(self.budget, self.backend.device.max_allocation_bytes)
        tile = max(1, min(rows, limit // (inner * 4)))
        if tile == rows:
            return self.backend.linear(x, self.tensor(name))
        if x.shape[0] != 1:
            raise ValueError("Tiled weight projection requires a single input row")
        result = self.backend.empty((1, rows))
        for start in range(0, rows, tile):
            stop = min(start + tile, rows)
            self.backend.copy(self.backend.linear(x, self.tensor(name, start, stop)), result,
                              target_offset=start)
        return result


class ReferenceModel:
    """Oracle token loop with the reference's public surface (model.py:36-357)."""

    def __init__(self, config, weights, *, backend, context_length=None,
                 weight_cache_bytes=256 * 1024 * 1024, record=False):
        self.config = config
        if context_length is None:
            context_length = min(2048, config.max_positions)
        if type(context_length) is not int or not 0 < context_length <= config.max_positions:
            raise ValueError(f"context_length must be in [1, {config.max_positions}]")
        self.weights = adapt_weights(config, weights)
        self.backend = backend
        self.context_length = context_length
        self.weight_cache = WeightCache(backend, self.weights, weight_cache_bytes)
        self.frequencies = backend.upload(config.inverse_frequencies())
        self.record = record
        self.reset()

    def reset(self):
        self.position, self._failed = 0, False
        self.states = [{} for _ in range(self.config.layers)]
        self.decisions = []     # per token: list of per-layer decision dicts

    # building blocks (model.py:79-93) ---------------------------------------------
    def _norm(self, x, name, width=None, eps=None):
        c = self.config
        gain = self.weight_cache.tensor(name) if name else None
        return self.backend.norm(x, gain, width or c.hidden_size, c.norm_eps if eps is None else eps)

    def _linear(self, x, name):
        return self.weight_cache.linear(x, name)

    def _ffn(self, x, root):
        b = self.backend
        return self._linear(b.swiglu(self._linear(x, root + "gate"), self._linear(x, root + "up")),
                            root + "down")

    def _rotate(self, x, positions, heads):
        return self.backend.rotate(x, self.frequencies, positions, heads, self.config.head_dim,
                                   self.config.split_half_rope)

    # grouped-query attention over a ring (model.py:95-116) ------------------------
    def _gqa(self, x, prefix, state, layer, position):
        b, c = self.backend, self.config
        kv_heads = c.layer_kv_heads(layer)
        query = self._linear(x, prefix + "q")
        key, value = self._linear(x, prefix + "k"), self._linear(x, prefix + "v")
        if c.qk_norm:
            query = self._norm(query, prefix + "q_norm", c.head_dim)
            key = self._norm(key, prefix + "k_norm", c.head_dim)
        query = self._rotate(query, position, c.query_heads)
        key = self._rotate(key, position, kv_heads)
        ring = state.get("ring")
        if ring is None:
            capacity = min(c.layer_window(layer) or self.context_length, self.context_length)
            ring = state["ring"] = Ring(b, capacity, kv_heads * c.head_dim)
        ring.append(b, key, value)
        relay = state.get("relay")
        attended = b.attention(query, ring.k, ring.v, heads=c.query_heads, kv_heads=kv_heads,
                               dim=c.head_dim, start=ring.start, length=ring.length,
                               extra_keys=relay.k if relay else None,
                               extra_values=relay.v if relay else None,
                               extra_length=relay.count if relay else 0)
        if c.family == "flashnano-1.6":
            self._update_cbr(x, prefix, state, kv_heads)
        return self._linear(attended, prefix + "o")

    # FlashNano 1.6 chunk summaries (model.py:118-144) -----------------------------
    def _update_cbr(self, x, prefix, state, kv_heads):
        b, c = self.backend, self.config
        if "pending" not in state:
            state["pending"] = b.empty((min(c.cbr_chunk_size, self.context_length), c.hidden_size))
        offset = self.position % c.cbr_chunk_size
        b.copy(x, state["pending"], target_offset=offset * c.hidden_size)
        if offset + 1 != c.cbr_chunk_size:
            return
        queries = self._norm(self.weight_cache.tensor(prefix + "cbr"), None, c.hidden_size, c.cbr_norm_eps)
        scores = b.empty((c.cbr_slots, c.cbr_chunk_size))
        b.run("pool_scores", (c.cbr_chunk_size, c.cbr_slots), state["pending"], queries, scores,
              c.cbr_chunk_size, c.cbr_slots, c.hidden_size)
        probs = b.softmax(scores)
        pooled, anchors = b.empty((c.cbr_slots, c.hidden_size)), b.empty((c.cbr_slots,))
        b.run("pool_mix", (c.hidden_size, c.cbr_slots), state["pending"], probs, pooled, anchors,
              c.cbr_chunk_size, c.cbr_slots, c.hidden_size, self.position + 1 - c.cbr_chunk_size)
        key, value = self._linear(pooled, prefix + "k"), self._linear(pooled, prefix + "v")
        key = self._rotate(self._norm(key, prefix + "k_norm", c.head_dim), anchors, kv_heads)
        relay = state.get("relay")
        if relay is None:
            capacity = (self.context_length // c.cbr_chunk_size) * c.cbr_slots
            relay = state["relay"] = Ring(b, capacity, kv_heads * c.head_dim)
        width = kv_heads * c.head_dim
        count = c.cbr_slots * width
        b.copy(key, relay.k, target_offset=relay.count * width, count=count)
        b.copy(value, relay.v, target_offset=relay.count * width, count=count)
        relay.count += c.cbr_slots
        if self.record:
            self._note("cbr_anchors", b.read(anchors).astype(np.int64).tolist())

    # FlashLighting latent attention (model.py:146-190) ----------------------------
    def _lighting(self, x, prefix, state, position):
        b, c = self.backend, self.config
        query = self._rotate(self._norm(self._linear(x, prefix + "q"), prefix + "q_norm", c.head_dim),
                             position, c.query_heads)
        latent = self._norm(self._linear(x, prefix + "latent"), prefix + "latent_norm", c.latent_dim)
        old = state.get("latent")
        n = 0 if old is None else old.shape[0]
        latents = b.empty((n + 1, c.latent_dim))
        if old is not None:
            b.copy(old, latents)
        b.copy(latent, latents, target_offset=n * c.latent_dim)
        positions = state.get("positions", []) + [self.position]
        counts = state.get("counts", []) + [1.0]
        key = self._norm(self._linear(latents, prefix + "k"), prefix + "k_norm", c.head_dim)
        key_positions = b.upload(np.asarray(positions, dtype=np.float32))
        key = self._rotate(key, key_positions, c.kv_heads)
        value = self._linear(latents, prefix + "v")
        scores = b.empty((c.query_heads, n + 1))
        b.run("scores", (n + 1, c.query_heads), query, key, key, scores, c.query_heads,
              c.kv_heads, c.head_dim, n + 1, 0, n + 1, 0)
        b.run("latent_mask", (n + 1, c.query_heads), scores, key_positions, c.query_heads,
              n + 1, state.get("memory_size", 0), self.position - c.window + 1)
        attended = b.mix(b.softmax(scores), value, c.query_heads, c.kv_heads, c.head_dim, 0, n + 1)
        overflow = max(0, n + 1 - c.window)
        if c.memory_slots == 0 and overflow:
            kept = b.empty((n + 1 - overflow, c.latent_dim))
            b.copy(latents, kept, source_offset=overflow * c.latent_dim)
            latents, positions, counts = kept, positions[overflow:], counts[overflow:]
            memory_size = 0
        elif overflow > c.memory_slots:
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
        if self.record:
            self._note("latent_positions", list(positions))
            self._note("memory_size", memory_size)
        return self._linear(attended, prefix + "o")

    # Heavy Medium sparse latent attention (model.py:192-229) ----------------------
    def _heavy_attention(self, x, prefix, state, position):
        b, c = self.backend, self.config
        query = self._norm(self._linear(x, prefix + "q"), None, c.head_dim, 1e-6)
        kv = self._linear(self._linear(x, prefix + "latent"), prefix + "kv_up")
        width = c.kv_heads * c.head_dim
        key, value = b.empty((1, width)), b.empty((1, width))
        b.copy(kv, key, count=width)
        b.copy(kv, value, source_offset=width, count=width)
        query = self._rotate(query, position, c.query_heads)
        key = self._rotate(self._norm(key, None, c.head_dim, 1e-6), position, c.kv_heads)
        ring = state.get("ring")
        if ring is None:
            ring = state["ring"] = Ring(b, self.context_length, width)
        ring.append(b, key, value)
        length = min(c.window, ring.count)
        start = ring.count - length
        geometry = c.source["long_context"]
        block = geometry["global_block_size"]
        blocks = (ring.count + block - 1) // block
        mean_keys, mean_values = b.empty((blocks, width)), b.empty((blocks, width))
        for src, dst in ((ring.k, mean_keys), (ring.v, mean_values)):
            b.run("block_means", (width, blocks), src, dst, ring.count, width, block)
        scores = b.empty((c.query_heads, length + blocks))
        b.run("scores", (length + blocks, c.query_heads), query, ring.k, mean_keys, scores,
              c.query_heads, c.kv_heads, c.head_dim, ring.capacity, start, length, blocks)
        host = b.read(scores)
        ends = np.minimum((np.arange(blocks) + 1) * block - 1, self.position)
        slope = np.float32(geometry.get("alibi_slope_scale", 0.015) / math.sqrt(c.head_dim))
        host[:, length:] -= slope * np.log1p((self.position - ends).astype(np.float32))
        slots = min(geometry["global_slots"], blocks)
        rank = np.argsort(-host[:, length:], axis=1, kind="stable")
        for h in range(c.query_heads):
            host[h, length + rank[h, slots:]] = -np.inf
        if self.record:
            self._note("topk_blocks", np.sort(rank[:, :slots], axis=1).tolist())
        attended = b.mix(b.softmax(b.upload(host)), ring.v, c.query_heads, c.kv_heads, c.head_dim,
                         start, length, mean_values, blocks)
        return self._linear(attended, prefix + "o")

    # Heavy Medium adaptive MoE (model.py:231-255) ----------------------------------
    def _moe(self, x, prefix):
        b, c, s = self.backend, self.config, self.config.source
        coarse = b.read(self._linear(x, prefix + "router.coarse.weight"))[0]
        fine = b.read(self._linear(x, prefix + "router.fine.weight"))[0]
        coarse += np.asarray(self.weights[prefix + "router.coarse.bias"]) + \
            np.asarray(self.weights[prefix + "router.group_bias"])
        fine += np.asarray(self.weights[prefix + "router.fine.bias"]) + \
            np.asarray(self.weights[prefix + "router.expert_bias"])
        experts, groups_n = s["routed_experts"], s["router_groups"]
        per_group = (experts + groups_n - 1) // groups_n
        group_of = np.minimum(np.arange(experts) // per_group, groups_n - 1)
        logits = (fine + coarse[group_of]) / np.float32(max(s.get("router_temperature", 1.0), 1e-4))
        probs = b.read(b.softmax(b.upload(logits.reshape(1, -1))))[0]
        max_k, min_k = s["router_top_k_max"], s["router_top_k_min"]
        order = np.argsort(-probs, kind="stable")[:max_k]
        chosen = probs[order].copy()
        confidence = chosen[0] - chosen[min(max_k - 1, 1)]
        entropy = -(probs * np.log(np.maximum(probs, np.float32(1e-9)))).sum()
        width_score = np.rint((np.float32(1) - confidence) * np.float32(2) +
                              entropy / max(np.float32(np.log(experts)), np.float32(1)))
        active = int(np.clip(min_k + width_score, min_k, max_k))
        chosen[active:] = 0
        chosen /= max(chosen.sum(), np.float32(1e-9))
        if self.record:
            self._note("experts", [int(e) for e in order[:active]])
            self._note("expert_weights", [float(w) for w in chosen[:active]])
        result = b.upload(np.zeros(x.shape, dtype=np.float32))
        for expert, weight in zip(order[:active], chosen[:active]):
            result = b.add(result, self._ffn(x, prefix + f"experts.{expert}."), float(weight))
        for shared in range(s["shared_experts"]):
            result = b.add(result, self._ffn(x, prefix + f"shared.{shared}."),
                           c.residual_scale / max(s["shared_experts"], 1))
        return result

    # one token (model.py:257-285) ---------------------------------------------------
    def _note(self, key, value):
        self._current.setdefault(key, []).append(value)

    def _step(self, token):
        b, c = self.backend, self.config
        hidden = b.upload(np.asarray(self.weights["embed"][token:token + 1], dtype=np.float32))
        position = b.upload(np.asarray([self.position], dtype=np.float32))
        token_record = []
        for layer, state in enumerate(self.states):
            prefix = f"layers.{layer}."
            self._current = {}
            if c.family == "heavy-medium-2.0":
                loops = state.setdefault("loops", [{} for _ in range(c.inner_loop_steps)])
                scale = c.residual_scale / math.sqrt(c.inner_loop_steps)
                for inner in loops:
                    attended = self._heavy_attention(self._norm(hidden, prefix + "a_norm"), prefix, inner,
                                                     position)
                    hidden = b.add(hidden, attended, scale)
                    hidden = b.add(hidden, self._moe(self._norm(hidden, prefix + "f_norm"), prefix), scale)
            elif c.family == "flashlighting-2.0":
                normalized = self._norm(hidden, prefix + "a_norm")
                attended = self._lighting(normalized, prefix, state, position)
                attention_gate = float(np.asarray(self.weights[prefix + "attention_gate"])[0])
                ffn_gate = float(np.asarray(self.weights[prefix + "ffn_gate"])[0])
                residual = b.add(b.upload(np.zeros(hidden.shape, dtype=np.float32)), attended, attention_gate)
                residual = b.add(residual, self._ffn(normalized, prefix + "ffn."), ffn_gate)
                hidden = b.add(hidden, residual, c.residual_scale)
            else:
                attended = self._gqa(self._norm(hidden, prefix + "a_norm"), prefix, state, layer, position)
                hidden = b.add(hidden, attended, c.residual_scale)
                hidden = b.add(hidden, self._ffn(self._norm(hidden, prefix + "f_norm"), prefix + "ffn."),
                               c.residual_scale)
            token_record.append(self._current)
        if self.record:
            self.decisions.append(token_record)
        self.position += 1
        return self._norm(hidden, "norm")

    # public token loop (model.py:287-357) -------------------------------------------
    def _tokens(self, ids):
        array = np.asarray(ids)
        if array.ndim != 1 or array.size == 0 or array.dtype.kind not in "iu":
            raise ValueError("input_ids must be a non-empty 1D integer sequence")
        if np.any(array < 0) or np.any(array >= self.config.vocab_size):
            raise ValueError("input token is outside the vocabulary")
        return array

    def prefill(self, input_ids, *, return_all=False):
        tokens = self._tokens(input_ids)
        if self._failed:
            raise RuntimeError("A previous device operation failed; call reset() before reusing this model")
        if self.position + len(tokens) > self.context_length:
            raise ValueError("input would exceed context_length; reset or allocate a larger context")
        out = []
        try:
            for i, token in enumerate(tokens):
                hidden = self._step(int(token))
                if return_all or i == len(tokens) - 1:
                    head = "embed" if self.config.tie_embeddings else "output"
                    out.append(self.backend.read(self._linear(hidden, head))[0])
        except Exception:
            self._failed = True
            raise
        return np.stack(out) if return_all else out[0]

    def decode(self, token_id):
        return self.prefill([token_id])

    def generate(self, input_ids, *, max_new_tokens=32, temperature=0.0, top_k=0, top_p=1.0,
                 seed=17, eos_token_id=None):
        tokens = self._tokens(input_ids)
        if type(max_new_tokens) is not int or max_new_tokens < 0:
            raise ValueError("max_new_tokens must be a non-negative integer")
        if not math.isfinite(temperature) or temperature < 0:
            raise ValueError("temperature must be finite and non-negative")
        if type(top_k) is not int or top_k < 0 or not math.isfinite(top_p) or not 0 < top_p <= 1:
            raise ValueError("top_k must be non-negative and top_p must be in (0,1]")
        eos = self.config.eos_token_id if eos_token_id is None else eos_token_id
        if type(eos) is not int or not 0 <= eos < self.config.vocab_size:
            raise ValueError("eos_token_id is outside vocabulary")
        if len(tokens) + max(0, max_new_tokens - 1) > self.context_length:
            raise ValueError("prompt plus requested generation exceeds context_length")
        self.reset()
        if max_new_tokens == 0:
            return []
        rng, generated = np.random.default_rng(seed), []
        logits = self.prefill(tokens)
        for i in range(max_new_tokens):
            if not np.all(np.isfinite(logits)):
                raise FloatingPointError("non-finite output logits")
            token = sample_next(logits, temperature, top_k, top_p, rng)
            generated.append(token)
            if token == eos or i + 1 == max_new_tokens:
                break
            logits = self.decode(token)
        return generated


def sample_next(logits, temperature, top_k, top_p, rng):
    """Greedy argmax or seeded top-k/top-p sampling (model.py:341-352)."""
    if temperature == 0:
        return int(np.argmax(logits))
    order = np.argsort(-logits, kind="stable")
    if top_k:
        order = order[:top_k]
    scores = logits[order].astype(np.float64) / temperature
    probs = np.exp(scores - scores.max())
    probs /= probs.sum()
    cutoff = min(len(order), int(np.searchsorted(np.cumsum(probs), top_p)) + 1)
    order, probs = order[:cutoff], probs[:cutoff]
    return int(rng.choice(order, p=probs / probs.sum()))
