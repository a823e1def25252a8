"""``MiracleModel``: the reference token-loop API on the CUDA engine.

Same public surface as the reference (miracle_reasoning/model.py:36-357):
``MiracleModel(config, weights, *, backend, context_length,
weight_cache_bytes)``, ``from_pretrained``, ``prefill(ids, return_all)``,
``decode(id)``, ``generate(...)``, ``reset()``, and the attributes
``position``, ``states`` and ``weight_cache``, with the same validation order
and error types.

What runs underneath is different: the checkpoint's stored bytes are copied
once into HBM (no LRU, no host widening).  For the grouped-query families
(flashnano-1.5/1.7, FlashLite) each token is one launch of the persistent
decode kernel (csrc/engine_kernel.cu) and greedy ``generate`` runs entirely on
the device (argmax feeds the next step).  FlashLighting without memory slots
runs on the same kernel (its latent cache as a key/value ring, see
``engine_plans``), and so do flashnano-1.6 (chunk relays pooled on the device
between steps) and FlashLighting with memory slots (rows that leave the window
absorbed into memory rows, the oldest two merged, on the device between steps;
csrc/aux_step.cuh); Heavy Medium runs its token step as device kernel launches
with the block top-k and expert routing on the GPU (csrc/heavy.cu).  Sampled
``generate`` reads the logits each step and samples on the host with the
reference's exact NumPy procedure.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import math
from pathlib import Path

import numpy as np

from . import _native
from .backend import CUDABackend
from .config import ModelConfig
from .weights import DTYPE_BF16, DTYPE_F32, SafeTensors, ShardedSafeTensors, adapt_weights, expected_shapes, \
    stored_tensor

_I32 = C.POINTER(C.c_int)
_F32 = C.POINTER(C.c_float)


def engine_config(config: ModelConfig, context_length: int) -> _native.ModelConfigC:
    """Flatten a ModelConfig into the C struct mr_model_config."""
    s = config.source
    c = _native.ModelConfigC()
    c.family = _native.FAMILY_CODES[config.family]
    for name in ("vocab_size", "hidden_size", "layers", "query_heads", "kv_heads", "head_dim", "ffn_dim",
                 "latent_dim", "memory_slots", "cbr_chunk_size", "cbr_slots", "inner_loop_steps"):
        setattr(c, name, getattr(config, name))
    c.context_length = context_length
    c.window = config.window or 0
    c.tie_embeddings = int(config.tie_embeddings)
    c.qk_norm = int(config.qk_norm)
    c.split_half_rope = int(config.split_half_rope)
    c.norm_eps, c.residual_scale, c.cbr_norm_eps = config.norm_eps, config.residual_scale, config.cbr_norm_eps
    if config.family == "heavy-medium-2.0":
        geometry = s["long_context"]
        c.routed_experts, c.router_groups = s["routed_experts"], s["router_groups"]
        c.router_top_k_min, c.router_top_k_max = s["router_top_k_min"], s["router_top_k_max"]
        c.shared_experts = s["shared_experts"]
        c.block_size, c.global_slots = geometry["global_block_size"], geometry["global_slots"]
        c.router_temperature = float(np.float32(max(s.get("router_temperature", 1.0), 1e-4)))
        c.alibi_slope = float(np.float32(geometry.get("alibi_slope_scale", 0.015) / math.sqrt(config.head_dim)))
    return c


class ResidentWeights:
    """Stands where the reference's WeightCache was: the whole model is resident."""

    def __init__(self, used, budget):
        self.used, self.budget = used, budget


class RingView:
    def __init__(self, count, capacity, length, start, width):
        self.count, self.capacity, self.width = count, capacity, width
        self.length, self.start = length, start


class RelayView:
    def __init__(self, count):
        self.count = count


class LatentView:
    def __init__(self, rows, width):
        self.shape = (rows, width)


def engine_plans(config):
    """Whether the device engine runs this configuration: every family does, given
    a FlashLighting attention window (the reference's latent mask needs one,
    model.py:165)."""
    return config.family != "flashlighting-2.0" or bool(config.window)


class RingDecisions:
    """FlashLighting's per-token latent decisions on the engine's ring (drop
    path): after the step at position p every layer keeps the latents of
    positions max(0, p + 1 - window) .. p and no memory rows.  Built on
    demand, in the format the reference records (one list per token of one dict per layer)."""

    def __init__(self, model):
        self._model = model

    def __len__(self):
        return self._model.position

    def __getitem__(self, t):
        if not 0 <= t < len(self):
            raise IndexError(t)
        c = self._model.config
        kept = list(range(max(0, t + 1 - c.window), t + 1))
        return [{"latent_positions": [list(kept)], "memory_size": [0]} for _ in range(c.layers)]


class MiracleModel:
    """FP32 next-token engine for six Miracle architectures on one B200.

    Each instance owns one sequence; call reset() for a new request.
    """

    def __init__(self, config, weights=None, *, backend=None, context_length=None,
                 weight_cache_bytes=256 * 1024 * 1024, tensor_parallel=None, record_decisions=False,
                 _synthetic=None):
        """``tensor_parallel=(rank, ranks, all_gather)``: this process decodes on one of
        ``ranks`` GPUs, each computing a slice of every projection's rows and of the
        KV heads (every rank makes the same calls in the same order; see
        mr_model_set_tensor_parallel).  ``record_decisions``: keep Heavy Medium's
        per-token top-k blocks and experts in ``decisions`` (each token then reads
        them back from the device)."""
        self.config = config
        if not engine_plans(config):
            raise ValueError("flashlighting-2.0 needs an attention window (window / local_window)")
        if context_length is None:
            context_length = min(2048, config.max_positions)
        if type(context_length) is not int or not 0 < context_length <= config.max_positions:
            raise ValueError(f"context_length must be in [1, {config.max_positions}]")
        if type(weight_cache_bytes) is not int or weight_cache_bytes < 4096:
            raise ValueError("weight_cache_bytes must be an integer >= 4096")
        # Validate the full checkpoint before creating any device allocations.
        self.weights = adapt_weights(config, weights) if _synthetic is None else None
        backend = backend if backend is not None else CUDABackend()
        if not isinstance(backend, CUDABackend):
            raise TypeError("MiracleModel runs on a CUDABackend (there is no CPU path)")
        self.backend = backend
        self.context_length = context_length
        self._handle = None
        kv = (C.c_int * config.layers)(*[config.layer_kv_heads(i) for i in range(config.layers)])
        windows = (C.c_int * config.layers)(*[config.layer_window(i) or 0 for i in range(config.layers)])
        inv = np.ascontiguousarray(config.inverse_frequencies(), dtype=np.float32)
        handle = C.c_void_p()
        cfg = engine_config(config, context_length)
        _native.call("mr_model_create", backend.context, C.byref(cfg), kv, windows,
                     inv.ctypes.data_as(_F32), C.byref(handle))
        self._handle = handle
        if _synthetic is None:
            self._load(self.weights)
        else:
            self._fill_synthetic(*_synthetic)
        self._ranks = 1
        if tensor_parallel is not None:
            rank, ranks, _ = tensor_parallel
            self._ranks = int(ranks)
            _native.call("mr_model_set_tensor_parallel", self._handle, int(rank), int(ranks))
        _native.call("mr_model_finalize", self._handle)
        if config.family == "heavy-medium-2.0":
            # the distance penalty's float32 log1p values, as the reference computes
            # them with NumPy (model.py:221-222), for every distance in the context
            table = np.ascontiguousarray(np.log1p(np.arange(context_length, dtype=np.float32)), dtype=np.float32)
            _native.call("mr_model_set_log1p_table", self._handle, table.ctypes.data_as(_F32), len(table))
        self.record_decisions = bool(record_decisions) and (
            config.family in ("heavy-medium-2.0", "flashnano-1.6")
            or (config.family == "flashlighting-2.0" and config.memory_slots > 0))
        self._decisions = []
        if tensor_parallel is not None and tensor_parallel[1] > 1:
            self._connect(*tensor_parallel)
        used = C.c_uint64()
        _native.call("mr_model_weight_bytes", self._handle, C.byref(used))
        self.weight_cache = ResidentWeights(int(used.value), weight_cache_bytes)
        self.frequencies = backend.upload(inv)
        self.reset()

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle and _native._lib is not None:
            _native._lib.mr_model_destroy(handle)
            self._handle = None

    def _connect(self, rank, ranks, all_gather):
        """Maps every rank's exchange arena: ``all_gather(bytes) -> [bytes of rank 0, ...]``
        is any host channel between the ranks (e.g. torch.distributed.all_gather_object)."""
        size = 64
        mine = (C.c_char * size)()
        _native.call("mr_model_tp_handle", self._handle, C.cast(mine, C.c_void_p), size)
        handles = all_gather(bytes(mine))
        if len(handles) != ranks or any(len(h) != size for h in handles):
            raise RuntimeError("tensor parallel: one handle per rank expected")
        joined = (C.c_char * (size * ranks)).from_buffer_copy(b"".join(handles))
        _native.call("mr_model_tp_connect", self._handle, C.cast(joined, C.c_void_p), size)

    def _load(self, weights):
        """Every tensor's stored bytes into HBM: read by the engine straight from a
        safetensors file when the mapping knows the tensor's file span, else copied
        from a host array."""
        span_of = getattr(weights, "file_span", None)
        for name, shape in expected_shapes(self.config).items():
            dims = (C.c_int64 * len(shape))(*shape)
            span = None
            if span_of is not None:
                try:
                    span = span_of(name)
                except (AttributeError, KeyError):
                    span = None
            if span is not None:
                path, offset, _, dtype = span
                _native.call("mr_model_load_file", self._handle, name.encode(), dtype, len(shape), dims,
                             os.fsencode(path), offset)
                continue
            dtype, array = stored_tensor(weights, name)
            _native.call("mr_model_load_tensor", self._handle, name.encode(), dtype, len(shape), dims,
                         array.ctypes.data)

    def _fill_synthetic(self, stored, seed):
        from . import synthetic
        host = synthetic.synthetic_weights(self.config, "F32", seed) if stored == "F32" else None
        for index, name, shape, std in synthetic.tensor_plan(self.config):
            dims = (C.c_int64 * len(shape))(*shape)
            if host is not None:
                array = np.ascontiguousarray(host[name], dtype=np.float32)
                _native.call("mr_model_load_tensor", self._handle, name.encode(), DTYPE_F32, len(shape), dims,
                             array.ctypes.data)
            elif std is None:
                _native.call("mr_model_fill_synthetic", self._handle, name.encode(), DTYPE_F32, len(shape), dims,
                             0, index, 0.0, 1.0)
            else:
                scale = float(np.float32(std / 65536.0))
                _native.call("mr_model_fill_synthetic", self._handle, name.encode(), DTYPE_BF16, len(shape), dims,
                             seed, index, scale, 0.0)

    @classmethod
    def synthetic(cls, config, *, stored="BF16", seed=0, **kwargs):
        """Random-initialised model built directly in HBM (see synthetic.py)."""
        return cls(config, None, _synthetic=(stored, seed), **kwargs)

    @classmethod
    def from_pretrained(cls, directory, *, family=None, **kwargs):
        directory = Path(directory)
        config = ModelConfig.from_dict(json.loads((directory / "config.json").read_text(encoding="utf-8")), family)
        if (directory / "model.safetensors").is_file():
            weights = SafeTensors(directory / "model.safetensors")
        elif (directory / "model.npz").is_file():
            weights = np.load(directory / "model.npz", allow_pickle=False)
        elif (directory / "model.safetensors.index.json").is_file():
            weights = ShardedSafeTensors(directory / "model.safetensors.index.json")
        else:
            raise ValueError("Expected model.safetensors, a safetensors index, or model.npz; "
                             "use the export command for PyTorch checkpoints")
        return cls(config, weights, **kwargs)

    # sequence state -------------------------------------------------------------
    def reset(self):
        """Release sequence caches while retaining weights."""
        _native.call("mr_model_reset", self._handle)
        self._decisions = []
        self._failed = False

    @property
    def position(self):
        value = C.c_int()
        _native.call("mr_model_position", self._handle, C.byref(value))
        return value.value

    @property
    def decisions(self):
        """Per token and layer, the discrete choices the reference records
        (heavy top-k blocks, MoE experts and weights, latent positions and memory size)."""
        if self.config.family == "flashlighting-2.0" and not self.config.memory_slots:
            return RingDecisions(self)
        return self._decisions

    def _read_decisions(self):
        """The last token's decisions per layer: Heavy Medium's top-k blocks and experts
        per loop; FlashLighting's latent positions and memory size after compaction."""
        c, s = self.config, self.config.source
        if c.family == "flashnano-1.6":  # chunk relays: no discrete choice to record
            self._decisions.append([{} for _ in range(c.layers)])
            return
        if c.family == "flashlighting-2.0":
            record = []
            for layer in range(c.layers):
                st = _native.LayerState()
                _native.call("mr_model_layer_state", self._handle, layer, 0, C.byref(st))
                record.append({"latent_positions": [self._latent_positions(layer, st.latent_rows)],
                               "memory_size": [st.memory_size]})
            self._decisions.append(record)
            return
        heads, slots, max_k = c.query_heads, s["long_context"]["global_slots"], s["router_top_k_max"]
        blocks = (C.c_int * max(heads * slots, 1))()
        experts, weights = (C.c_int * max_k)(), (C.c_float * max_k)()
        record = []
        for layer in range(c.layers):
            entry = {"topk": [], "experts": [], "expert_weights": []}
            for loop in range(c.inner_loop_steps):
                _native.call("mr_model_last_topk", self._handle, layer, loop, blocks, heads * slots)
                entry["topk"].append([[b for b in blocks[h * slots:(h + 1) * slots] if b >= 0] for h in range(heads)])
                _native.call("mr_model_last_experts", self._handle, layer, loop, experts, weights, max_k)
                chosen = [e for e in experts[:max_k] if e >= 0]
                entry["experts"].append(chosen)
                entry["expert_weights"].append([float(np.float32(w)) for w in weights[:len(chosen)]])
            record.append(entry)
        self._decisions.append(record)

    @property
    def states(self):
        """Per-layer cache views with the attributes the reference exposes."""
        c = self.config
        views = []
        for layer in range(c.layers):
            entry = {}
            loops = c.inner_loop_steps if c.family == "heavy-medium-2.0" else 1
            per_loop = []
            for loop in range(loops):
                st = _native.LayerState()
                _native.call("mr_model_layer_state", self._handle, layer, loop, C.byref(st))
                per_loop.append(st)
            st = per_loop[0]
            if st.present:
                width = c.layer_kv_heads(layer) * c.head_dim
                if c.family == "heavy-medium-2.0":
                    entry["loops"] = [{"ring": RingView(s.ring_count, s.ring_capacity, s.ring_length,
                                                        s.ring_start, c.kv_heads * c.head_dim)} for s in per_loop]
                elif c.family == "flashlighting-2.0":
                    entry["latent"] = LatentView(st.latent_rows, c.latent_dim)
                    entry["memory_size"] = st.memory_size
                    entry["positions"] = self._latent_positions(layer, st.latent_rows)
                    entry["counts"] = self._latent_counts(layer, st.latent_rows)
                else:
                    entry["ring"] = RingView(st.ring_count, st.ring_capacity, st.ring_length, st.ring_start, width)
                    if c.family == "flashnano-1.6" and st.relay_count:
                        entry["relay"] = RelayView(st.relay_count)
            views.append(entry)
        return views

    def _latent_positions(self, layer, rows):
        out = (C.c_int * max(rows, 1))()
        n = C.c_int()
        _native.call("mr_model_latent_positions", self._handle, layer, out, max(rows, 1), C.byref(n))
        return list(out[:n.value])

    def _latent_counts(self, layer, rows):
        out = (C.c_float * max(rows, 1))()
        n = C.c_int()
        _native.call("mr_model_latent_counts", self._handle, layer, out, max(rows, 1), C.byref(n))
        return [float(v) for v in out[:n.value]]

    # token loop -------------------------------------------------------------------
    def _tokens(self, ids):
        array = np.asarray(ids)
        if array.ndim != 1 or array.size == 0 or array.dtype.kind not in "iu":
            raise ValueError("input_ids must be a non-empty 1D integer sequence")
        if np.any(array < 0) or np.any(array >= self.config.vocab_size):
            raise ValueError("input token is outside the vocabulary")
        return array

    def prefill(self, input_ids, *, return_all=False):
        """Append a prompt, returning [vocab] or, if requested, [tokens, vocab]."""
        tokens = self._tokens(input_ids)
        if self._failed:
            raise RuntimeError("A previous device operation failed; call reset() before reusing this model")
        if self.position + len(tokens) > self.context_length:
            raise ValueError("input would exceed context_length; reset or allocate a larger context")
        ids = np.ascontiguousarray(tokens, dtype=np.int32)
        V = self.config.vocab_size
        out = np.empty((len(ids), V) if return_all else (V,), dtype=np.float32)
        try:
            if self.record_decisions:
                for i in range(len(ids)):
                    row = np.empty(V, dtype=np.float32)
                    _native.call("mr_model_prefill", self._handle, ids[i:].ctypes.data_as(_I32), 1, 0,
                                 row.ctypes.data_as(_F32))
                    self._read_decisions()
                    if return_all:
                        out[i] = row
                    elif i == len(ids) - 1:
                        out[:] = row
            else:
                _native.call("mr_model_prefill", self._handle, ids.ctypes.data_as(_I32), len(ids), int(return_all),
                             out.ctypes.data_as(_F32))
        except Exception:
            self._failed = True
            raise
        return out

    def decode(self, token_id):
        """Append one token to the current sequence and return next-token logits."""
        V = self.config.vocab_size
        if (type(token_id) is int and 0 <= token_id < V and not self.record_decisions
                and not self._failed and self.position < self.context_length):
            # the common case, without building and checking an id array (prefill's checks
            # would all pass): one token straight to the C entry point
            out = np.empty(V, dtype=np.float32)
            try:
                _native.call("mr_model_prefill", self._handle, C.byref(C.c_int(token_id)), 1, 0,
                             out.ctypes.data_as(_F32))
            except Exception:
                self._failed = True
                raise
            return out
        return self.prefill([token_id])

    def generate(self, input_ids, *, max_new_tokens=32, temperature=0.0, top_k=0, top_p=1.0, seed=17,
                 eos_token_id=None):
        """Return generated token IDs, excluding the prompt and including EOS."""
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
        if not self.record_decisions and self._ranks == 1 and (temperature > 0 or self.config.family == "heavy-medium-2.0"):
            # sampling (and Heavy Medium's argmax) on the device, the reference's procedure to the bit
            return self._generate_on_device(tokens, max_new_tokens, eos, float(temperature), int(top_k),
                                            float(top_p), np.random.default_rng(seed))
        if temperature == 0 and not self.record_decisions:
            return self._generate_greedy(tokens, max_new_tokens, eos)
        rng, generated = np.random.default_rng(seed), []
        logits = self.prefill(tokens)
        for i in range(max_new_tokens):
            if not np.all(np.isfinite(logits)):
                raise FloatingPointError("non-finite output logits")
            token = int(np.argmax(logits)) if temperature == 0 else sample_next(logits, temperature, top_k, top_p, rng)
            generated.append(token)
            if token == eos or i + 1 == max_new_tokens:
                break
            logits = self.decode(token)
        return generated

    def _generate_on_device(self, tokens, max_new_tokens, eos, temperature, top_k, top_p, rng):
        state = rng.bit_generator.state["state"]
        mask = (1 << 64) - 1
        pcg = (C.c_uint64 * 4)(state["state"] >> 64, state["state"] & mask, state["inc"] >> 64, state["inc"] & mask)
        ids = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(max_new_tokens, dtype=np.int32)
        count, nonfinite = C.c_int(), C.c_int()
        try:
            _native.call("mr_model_generate_sampled", self._handle, ids.ctypes.data_as(_I32), len(ids),
                         max_new_tokens, eos, temperature, top_k, top_p, pcg, out.ctypes.data_as(_I32),
                         C.byref(count), C.byref(nonfinite))
        except Exception:
            self._failed = True
            raise
        if nonfinite.value:  # as the reference, which raises without latching (model.py:331-332)
            raise FloatingPointError("non-finite output logits")
        return [int(t) for t in out[:count.value]]

    def _generate_greedy(self, tokens, max_new_tokens, eos):
        ids = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(max_new_tokens, dtype=np.int32)
        count, nonfinite = C.c_int(), C.c_int()
        try:
            _native.call("mr_model_generate_greedy", self._handle, ids.ctypes.data_as(_I32), len(ids),
                         max_new_tokens, eos, out.ctypes.data_as(_I32), C.byref(count), C.byref(nonfinite))
        except Exception:
            self._failed = True
            raise
        if nonfinite.value:
            raise FloatingPointError("non-finite output logits")
        return [int(t) for t in out[:count.value]]


def sample_next(logits, temperature, top_k, top_p, rng):
    """Seeded top-k/top-p sampling, the reference's exact procedure (model.py:343-352)."""
    order = np.argsort(-logits, kind="stable")
    if top_k:
        order = order[:top_k]
    scores = logits[order].astype(np.float64) / temperature
    probs = np.exp(scores - scores.max())
    probs /= probs.sum()
    cutoff = min(len(order), int(np.searchsorted(np.cumsum(probs), top_p)) + 1)
    order, probs = order[:cutoff], probs[:cutoff]
    return int(rng.choice(order, p=probs / probs.sum()))
