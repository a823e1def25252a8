"""Checkpoint reading, name adaptation and shape validation (host side).

Keeps the reference's loading semantics (miracle_reasoning/weights.py):
memory-mapped F32/F16/BF16 safetensors with the same header checks (14-61),
BF16 widened by ``u16 << 16`` (64-74), sharded indexes with path containment
(77-99), the native-checkpoint name tables (145-208), the expected shape table
(211-245) and validation of every tensor before any device allocation
(248-255).

What changes is residency: the reference widens each weight to float32 on the
host and keeps a budgeted LRU of device copies (weights.py:258-297).  Here each
tensor's STORED bytes (F32, F16 or BF16) are handed once to the CUDA engine,
which keeps the whole model resident in HBM and widens in registers.
``stored_tensor`` returns those raw bytes without widening.
"""
from __future__ import annotations

import json
import math
import struct
from collections.abc import Mapping
from pathlib import Path

import numpy as np

# dtype codes shared with include/miracle_cuda.h (MR_DTYPE_*)
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
_SAFETENSORS_TYPES = {"F32": ("<f4", DTYPE_F32), "F16": ("<f2", DTYPE_F16), "BF16": ("<u2", DTYPE_BF16)}
_MAX_HEADER = 100_000_000


class SafeTensors(Mapping):
    """Memory-mapped F32/F16/BF16 safetensors file (no PyTorch needed)."""

    def __init__(self, path):
        self.path = Path(path)
        size = self.path.stat().st_size
        with self.path.open("rb") as handle:
            prefix = handle.read(8)
            if len(prefix) != 8:
                raise ValueError("Truncated safetensors header")
            (length,) = struct.unpack("<Q", prefix)
            if length > min(_MAX_HEADER, size - 8):
                raise ValueError("Invalid safetensors header length")
            metadata = json.loads(handle.read(length))
        self.offset = 8 + length
        self.entries = {}
        spans = []
        for name, entry in metadata.items():
            if name == "__metadata__":
                continue
            kind = entry["dtype"]
            if kind not in _SAFETENSORS_TYPES:
                raise ValueError(f"Unsupported weight dtype {kind} in {name}; export to FP32 first")
            shape, offsets = entry["shape"], entry["data_offsets"]
            if not isinstance(shape, list) or any(type(n) is not int or n < 0 for n in shape):
                raise ValueError(f"Invalid shape for {name}")
            if len(offsets) != 2 or any(type(n) is not int for n in offsets):
                raise ValueError(f"Invalid offsets for {name}")
            start, end = offsets
            numpy_type = _SAFETENSORS_TYPES[kind][0]
            if start < 0 or end - start != math.prod(shape) * np.dtype(numpy_type).itemsize \
                    or end > size - self.offset:
                raise ValueError(f"Invalid safetensors extent for {name}")
            self.entries[name] = (tuple(shape), kind, numpy_type, start)
            spans.append((start, end))
        spans.sort()
        if any(later[0] < earlier[1] for earlier, later in zip(spans, spans[1:])):
            raise ValueError("Overlapping safetensors data")

    def __iter__(self):
        return iter(self.entries)

    def __len__(self):
        return len(self.entries)

    def raw(self, key):
        shape, _, numpy_type, start = self.entries[key]
        return np.memmap(self.path, mode="r", offset=self.offset + start, dtype=numpy_type, shape=shape)

    def __getitem__(self, key):
        data = self.raw(key)
        return BF16Array(data) if self.entries[key][1] == "BF16" else data


class BF16Array:
    """BF16 storage (uint16 bits) widened to float32 only where indexed."""

    def __init__(self, data):
        self.data, self.shape = data, data.shape

    def __getitem__(self, key):
        return (np.asarray(self.data[key], dtype=np.uint32) << 16).view(np.float32)

    def __array__(self, dtype=None, copy=None):
        widened = self[:]
        return widened.astype(dtype, copy=False) if dtype is not None else widened


class ShardedSafeTensors(Mapping):
    """``model.safetensors.index.json`` over several safetensors files."""

    def __init__(self, index):
        index = Path(index)
        self.names = json.loads(index.read_text(encoding="utf-8"))["weight_map"]
        root = index.parent.resolve()
        self.shards = {}
        for filename in set(self.names.values()):
            path = (root / filename).resolve()
            if not path.is_relative_to(root):
                raise ValueError("Safetensors shard path escapes the model directory")
            self.shards[filename] = SafeTensors(path)
        for key, filename in self.names.items():
            if key not in self.shards[filename]:
                raise ValueError(f"Shard {filename} does not contain {key}")

    def __iter__(self):
        return iter(self.names)

    def __len__(self):
        return len(self.names)

    def __getitem__(self, key):
        return self.shards[self.names[key]][key]


class AliasedWeights(Mapping):
    """Canonical names resolved through a native-checkpoint name table."""

    def __init__(self, original, names):
        self.original, self.names = original, names
        missing = [v for v in names.values() if v not in original]
        if missing:
            raise ValueError(f"Missing checkpoint tensors: {', '.join(missing[:12])}")

    def __iter__(self):
        return iter(self.names)

    def __len__(self):
        return len(self.names)

    def __getitem__(self, key):
        return self.original[self.names[key]]


def save_safetensors(path, arrays, dtype="F32"):
    """Write tensors sequentially as F32 (default) or BF16/F16, 16 MiB at a time.

    BF16 output rounds float32 to nearest-even; arrays that already hold BF16
    bits (``BF16Array``) are written bit-for-bit.
    """
    itemsize = {"F32": 4, "F16": 2, "BF16": 2}[dtype]
    header, offset = {}, 0
    for key, value in arrays.items():
        length = math.prod(value.shape) * itemsize
        header[key] = {"dtype": dtype, "shape": list(value.shape), "data_offsets": [offset, offset + length]}
        offset += length
    encoded = json.dumps(header, separators=(",", ":")).encode()
    encoded += b" " * (-len(encoded) % 8)
    with Path(path).open("wb") as handle:
        handle.write(struct.pack("<Q", len(encoded)))
        handle.write(encoded)
        for value in arrays.values():
            if not value.shape:
                handle.write(_encode(np.asarray(value), dtype).tobytes())
                continue
            row_bytes = max(math.prod(value.shape[1:]) * 4, 1)
            tile = max(1, 16 * 1024 * 1024 // row_bytes)
            for start in range(0, value.shape[0], tile):
                if dtype == "BF16" and isinstance(value, BF16Array):
                    block = np.asarray(value.data[start:start + tile], dtype="<u2")
                else:
                    block = _encode(np.asarray(value[start:start + tile], dtype="<f4"), dtype)
                handle.write(memoryview(np.ascontiguousarray(block)).cast("B"))


def _encode(array, dtype):
    array = np.asarray(array, dtype="<f4")
    if dtype == "F32":
        return array
    if dtype == "F16":
        return array.astype("<f2")
    return float32_to_bf16_bits(array)


def float32_to_bf16_bits(array):
    """Round float32 to bfloat16 (nearest-even) and return the uint16 bits."""
    bits = np.ascontiguousarray(array, dtype=np.float32).view(np.uint32)
    rounded = bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    out = (rounded >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(array)
    if np.any(nan):
        out[nan] = ((bits[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return out


def stored_tensor(weights, name):
    """(dtype code, contiguous array of the stored bytes) for ``weights[name]``.

    BF16 comes back as its uint16 bits, F16 as float16, everything else as
    float32 (float64 NumPy input is narrowed the way the reference narrows it,
    ``np.ascontiguousarray(..., float32)``).
    """
    value = weights[name]
    if isinstance(value, BF16Array):
        return DTYPE_BF16, np.ascontiguousarray(value.data, dtype=np.uint16)
    if getattr(value, "dtype", None) is not None and np.dtype(value.dtype) == np.float16:
        return DTYPE_F16, np.ascontiguousarray(value, dtype=np.float16)
    return DTYPE_F32, np.ascontiguousarray(np.asarray(value, dtype=np.float32))


# native checkpoint names (weights.py:145-208) -------------------------------------
_LAYER_ROOTS = {
    # family: (layer root fmt, attention norm, ffn norm, attention module, ffn module)
    "flashnano-1.5": ("backbone.layers.{i}.", "input_norm.weight", "post_attention_norm.weight",
                      "attention.", "feed_forward."),
    "flashlite-2.0": ("backbone.layers.{i}.", "input_norm.weight", "post_attention_norm.weight",
                      "attention.", "feed_forward."),
    "flashnano-1.6": ("blocks.{i}.", "attn_norm.weight", "ffn_norm.weight", "attn.", "ffn."),
    "flashnano-1.7": ("blocks.{i}.", "attn_norm_weight", "ffn_norm_weight", "attn.", "ffn."),
    "flashlighting-2.0": ("layers.{i}.", "input_norm.weight", None, "attention.", "feed_forward."),
    "heavy-medium-2.0": ("blocks.{i}.", "attention_norm.weight", "moe_norm.weight", "attention.", None),
}
_EMBED = {"flashnano-1.5": "backbone.token_embedding.weight", "flashlite-2.0": "backbone.embed_tokens.weight",
          "flashlighting-2.0": "embed_tokens.weight"}
_FINAL_NORM = {"flashnano-1.5": "backbone.norm.weight", "flashlite-2.0": "backbone.norm.weight",
               "flashnano-1.7": "final_norm_weight"}


def native_names(config):
    """Canonical name -> name in the family's native training checkpoint."""
    c, fam = config, config.family
    nano16 = fam == "flashnano-1.6"
    names = {"embed": _EMBED.get(fam, "embedding.weight"), "norm": _FINAL_NORM.get(fam, "final_norm.weight")}
    if not c.tie_embeddings:
        names["output"] = "lm_head.weight"
    root_fmt, attn_norm, ffn_norm, attn, ffn = _LAYER_ROOTS[fam]
    for i in range(c.layers):
        p, root = f"layers.{i}.", root_fmt.format(i=i)
        names[p + "a_norm"] = root + attn_norm
        if ffn_norm:
            names[p + "f_norm"] = root + ffn_norm
        names[p + "q"] = root + attn + ("w_q.weight" if nano16 else "q_proj.weight")
        out = "w_o.weight" if nano16 else "out_proj.weight" if fam == "heavy-medium-2.0" else "o_proj.weight"
        names[p + "o"] = root + attn + out
        if fam in ("flashlighting-2.0", "heavy-medium-2.0"):
            names[p + "latent"] = root + attn + "kv_down.weight"
            if fam == "flashlighting-2.0":
                names[p + "latent_norm"] = root + attn + "kv_norm.weight"
                names[p + "k"] = root + attn + "k_up.weight"
                names[p + "v"] = root + attn + "v_up.weight"
                names[p + "attention_gate"] = root + "attention_gate"
                names[p + "ffn_gate"] = root + "ffn_gate"
            else:
                names[p + "kv_up"] = root + attn + "kv_up.weight"
        else:
            for key in ("k", "v"):
                names[p + key] = root + attn + (f"w_{key}.weight" if nano16 else f"{key}_proj.weight")
        if c.qk_norm and fam != "heavy-medium-2.0":
            for key in ("q", "k"):
                native = f"qk_norm_{key}" if fam == "flashnano-1.7" else f"{key}_norm.weight"
                names[p + key + "_norm"] = root + attn + native
        if ffn:
            for key in ("gate", "up", "down"):
                names[p + "ffn." + key] = root + ffn + (f"w_{key}.weight" if nano16 else f"{key}_proj.weight")
        if nano16:
            names[p + "cbr"] = root + "cbr.queries"
        if fam == "heavy-medium-2.0":
            for level in ("coarse", "fine"):
                for key in ("weight", "bias"):
                    names[p + f"router.{level}.{key}"] = root + f"moe.router.{level}.{key}"
            for key in ("group_bias", "expert_bias"):
                names[p + "router." + key] = root + "moe.router." + key
            for ei in range(c.source["routed_experts"]):
                for key in ("gate", "up", "down"):
                    names[p + f"experts.{ei}.{key}"] = root + f"moe.experts.expert_{ei}.{key}_weight"
            for ei in range(c.source["shared_experts"]):
                for key in ("gate", "up", "down"):
                    names[p + f"shared.{ei}.{key}"] = root + f"moe.shared_experts.{ei}.{key}_weight"
    return names


def expected_shapes(c):
    """Canonical name -> required shape, in the reference's enumeration order."""
    h, d, q, f = c.hidden_size, c.head_dim, c.query_heads * c.head_dim, c.ffn_dim
    heavy = c.family == "heavy-medium-2.0"
    shapes = {"embed": (c.vocab_size, h), "norm": (h,)}
    if not c.tie_embeddings:
        shapes["output"] = (c.vocab_size, h)
    for i in range(c.layers):
        p, kv = f"layers.{i}.", c.layer_kv_heads(i) * d
        shapes.update({p + "a_norm": (h,), p + "q": (q, h), p + "o": (h, q)})
        if c.family != "flashlighting-2.0":
            shapes[p + "f_norm"] = (h,)
        if c.latent_dim:
            shapes[p + "latent"] = (c.latent_dim, h)
        if heavy:
            shapes[p + "kv_up"] = (2 * kv, c.latent_dim)
            experts, groups = c.source["routed_experts"], c.source["router_groups"]
            for level, n in (("coarse", groups), ("fine", experts)):
                shapes[p + f"router.{level}.weight"] = (n, h)
                shapes[p + f"router.{level}.bias"] = (n,)
            shapes[p + "router.group_bias"] = (groups,)
            shapes[p + "router.expert_bias"] = (experts,)
        else:
            inner = c.latent_dim or h
            shapes.update({p + "k": (kv, inner), p + "v": (kv, inner)})
            if c.qk_norm:
                shapes.update({p + "q_norm": (d,), p + "k_norm": (d,)})
        if c.family == "flashlighting-2.0":
            shapes.update({p + "latent_norm": (c.latent_dim,), p + "attention_gate": (1,), p + "ffn_gate": (1,)})
        if c.family == "flashnano-1.6":
            shapes[p + "cbr"] = (c.cbr_slots, h)
        if heavy:
            roots = [p + f"experts.{e}." for e in range(c.source["routed_experts"])]
            roots += [p + f"shared.{e}." for e in range(c.source["shared_experts"])]
        else:
            roots = [p + "ffn."]
        for root in roots:
            shapes.update({root + "gate": (f, h), root + "up": (f, h), root + "down": (h, f)})
    return shapes


def adapt_weights(config, original):
    """Resolve native names when needed and check every tensor's shape."""
    weights = original if "embed" in original else AliasedWeights(original, native_names(config))
    for key, shape in expected_shapes(config).items():
        if key not in weights:
            raise ValueError(f"Missing tensor {key}")
        if weights[key].shape != shape:
            raise ValueError(f"{key}: expected {shape}, got {weights[key].shape}")
    return weights
