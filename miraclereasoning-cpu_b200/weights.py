"""Checkpoint reading, name adaptation and shape validation (host side).

Loading semantics are the reference's (miracle_reasoning/weights.py): F32,
F16 and BF16 safetensors only, the header checked before anything is read
(14-61), BF16 widened exactly to float32 where float32 values are asked for
(64-74), sharded indexes whose files must stay inside the model directory
(77-99), native-checkpoint name tables (145-208), the expected shape table
(211-245), and every tensor validated before any device allocation (248-255).

Residency differs: the reference widens each weight to float32 on the host
and keeps a budgeted LRU of device copies (weights.py:258-297).  Here each
tensor's STORED bytes go to the CUDA engine once and stay resident in HBM.
For a safetensors checkpoint the engine reads them itself, straight from the
file into HBM through page-locked double buffers (``file_span`` gives it the
file, offset and size; ``mr_model_load_file``); other mappings hand over a
host array of the stored bytes (``stored_tensor``).
"""
from __future__ import annotations

import json
import math
import os
import struct
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path

import numpy as np

# dtype codes shared with include/miracle_cuda.h (MR_DTYPE_*)
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
# safetensors dtype -> (little-endian NumPy storage type, engine dtype code)
_STORAGE = {"F32": ("<f4", DTYPE_F32), "F16": ("<f2", DTYPE_F16), "BF16": ("<u2", DTYPE_BF16)}
_HEADER_LIMIT = 100_000_000


@dataclass(frozen=True)
class TensorEntry:
    """One tensor of a safetensors file: its stored kind, shape and byte span
    [begin, end) relative to the start of the data section."""
    kind: str
    shape: tuple
    begin: int
    end: int

    @property
    def storage(self):
        return np.dtype(_STORAGE[self.kind][0])

    @property
    def code(self):
        return _STORAGE[self.kind][1]


def _fail(message):
    raise ValueError(message)


def read_safetensors_header(path):
    """(offset of the data section, {name: TensorEntry}) of a safetensors file,
    after checking everything the loader relies on: the header length, the
    dtypes, shapes and offsets, that every span lies inside the file and
    matches its shape, and that no two spans overlap."""
    size = os.path.getsize(path)
    with open(path, "rb") as handle:
        head = handle.read(8)
        if len(head) < 8:
            _fail("Truncated safetensors header")
        header_bytes = struct.unpack("<Q", head)[0]
        if header_bytes > min(_HEADER_LIMIT, size - 8):
            _fail("Invalid safetensors header length")
        header = json.loads(handle.read(header_bytes))
    data_start, data_size = 8 + header_bytes, size - 8 - header_bytes
    entries = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        kind = info["dtype"]
        if kind not in _STORAGE:
            _fail(f"Unsupported weight dtype {kind} in {name}; export to FP32 first")
        shape, span = info["shape"], info["data_offsets"]
        if not isinstance(shape, list) or not all(type(n) is int and n >= 0 for n in shape):
            _fail(f"Invalid shape for {name}")
        if len(span) != 2 or not all(type(n) is int for n in span):
            _fail(f"Invalid offsets for {name}")
        entry = TensorEntry(kind, tuple(shape), span[0], span[1])
        if entry.begin < 0 or entry.end > data_size or \
                entry.end - entry.begin != math.prod(entry.shape) * entry.storage.itemsize:
            _fail(f"Invalid safetensors extent for {name}")
        entries[name] = entry
    ordered = sorted(entries.values(), key=lambda e: (e.begin, e.end))
    for left, right in zip(ordered, ordered[1:]):
        if right.begin < left.end:
            _fail("Overlapping safetensors data")
    return data_start, entries


class BF16Array:
    """BF16 weights kept as their uint16 bits; the rows asked for come back as
    float32 (bits << 16, exact)."""

    def __init__(self, bits):
        self.data = bits
        self.shape = bits.shape

    def __getitem__(self, index):
        widened = np.left_shift(np.asarray(self.data[index], dtype=np.uint32), np.uint32(16))
        return widened.view(np.float32)

    def __array__(self, dtype=None, copy=None):
        values = self[...]
        return values if dtype is None else values.astype(dtype, copy=False)


class SafeTensors(Mapping):
    """A safetensors file: stored-dtype views of one read-only memory map of
    its data section (BF16 tensors as ``BF16Array``)."""

    def __init__(self, path):
        self.path = Path(path)
        self._data_start, self.entries = read_safetensors_header(self.path)
        self._map = None

    def __iter__(self):
        return iter(self.entries)

    def __len__(self):
        return len(self.entries)

    def _bytes(self):
        if self._map is None:
            data_size = os.path.getsize(self.path) - self._data_start
            self._map = np.memmap(self.path, mode="r", dtype=np.uint8, offset=self._data_start,
                                  shape=(data_size,)) if data_size else np.zeros(0, np.uint8)
        return self._map

    def raw(self, name):
        """The tensor in its stored dtype (uint16 bits for BF16), not widened."""
        entry = self.entries[name]
        return self._bytes()[entry.begin:entry.end].view(entry.storage).reshape(entry.shape)

    def __getitem__(self, name):
        values = self.raw(name)
        return BF16Array(values) if self.entries[name].kind == "BF16" else values

    def file_span(self, name):
        """(path, absolute byte offset, byte count, engine dtype code) of a tensor."""
        entry = self.entries[name]
        return str(self.path), self._data_start + entry.begin, entry.end - entry.begin, entry.code


class ShardedSafeTensors(Mapping):
    """``model.safetensors.index.json``: every name served by the shard file
    the index assigns it, each shard inside the index's directory."""

    def __init__(self, index):
        index = Path(index)
        weight_map = json.loads(index.read_text(encoding="utf-8"))["weight_map"]
        root = index.parent.resolve()
        files = {}
        for filename in sorted(set(weight_map.values())):
            path = (root / filename).resolve()
            if os.path.commonpath([root, path]) != str(root):
                _fail("Safetensors shard path escapes the model directory")
            files[filename] = SafeTensors(path)
        self._where = {}
        for name, filename in weight_map.items():
            if name not in files[filename]:
                _fail(f"Shard {filename} does not contain {name}")
            self._where[name] = files[filename]
        self.names, self.shards = weight_map, files

    def __iter__(self):
        return iter(self._where)

    def __len__(self):
        return len(self._where)

    def __getitem__(self, name):
        return self._where[name][name]

    def file_span(self, name):
        return self._where[name].file_span(name)


class AliasedWeights(Mapping):
    """Canonical names over a checkpoint that uses its training code's names
    (the native name tables below); every aliased tensor must exist."""

    def __init__(self, original, names):
        absent = [native for native in names.values() if native not in original]
        if absent:
            _fail(f"Missing checkpoint tensors: {', '.join(absent[:12])}")
        self.original, self.names = original, names

    def __iter__(self):
        return iter(self.names)

    def __len__(self):
        return len(self.names)

    def __getitem__(self, name):
        return self.original[self.names[name]]

    def file_span(self, name):
        if not hasattr(self.original, "file_span"):
            raise AttributeError("file_span")
        return self.original.file_span(self.names[name])


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
