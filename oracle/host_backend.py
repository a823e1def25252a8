"""Host execution of the reference kernel set behind the ``OpenCLBackend`` surface.

TEST INFRASTRUCTURE ONLY: the checker the CUDA product is compared against.
Nothing in the product package imports this module.

``HostBackend`` offers the method surface of the reference backend
(miracle_reasoning/opencl.py:129-303): ``empty/upload/read/copy/run/linear/
norm/rotate/add/swiglu/softmax/attention/mix/finish`` and ``.device`` with
``max_allocation_bytes``.  "Device memory" is host float32 NumPy storage and
every ``run`` evaluates one NDRange through one of two kernel libraries:

* ``kernels="oracle"`` — the plain-C restatement (oracle/kernels.c);
* ``kernels="reference"`` — the reference's own kernels.cl compiled on the host
  (oracle/_ref/libref_kernels.so, see oracle/ref_host.cpp).

Argument marshalling follows opencl.py:219-239: Tensor -> pointer, Python/NumPy
float -> float32, int in int32 range -> int32, anything else is rejected.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import build as _build

_P, _I, _F = "p", "i", "f"
# Kernel name -> (NDRange rank, argument kinds) in kernels.cl argument order.
SIGNATURES = {
    "linear": (2, (_P, _P, _P, _I, _I, _I)),
    "rms": (1, (_P, _P, _P, _I, _I, _F, _I)),
    "rope": (1, (_P, _P, _P, _P, _I, _I, _I, _I)),
    "swiglu": (1, (_P, _P, _P, _I)),
    "axpy": (1, (_P, _P, _P, _I, _F)),
    "scores": (2, (_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I)),
    "softmax": (1, (_P, _P, _I, _I)),
    "latent_mask": (2, (_P, _P, _I, _I, _I, _I)),
    "mix": (1, (_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I)),
    "pool_scores": (2, (_P, _P, _P, _I, _I, _I)),
    "pool_mix": (2, (_P, _P, _P, _P, _I, _I, _I, _I)),
    "merge_rows": (1, (_P, _P, _I, _F, _F)),
    "block_means": (2, (_P, _P, _I, _I, _I)),
}
_CTYPE = {_P: C.c_void_p, _I: C.c_int, _F: C.c_float}


class HostError(RuntimeError):
    pass


def load_kernels(kind: str = "oracle"):
    """Return (ctypes library, symbol prefix) for ``kind`` in {oracle, reference}."""
    if kind == "oracle":
        path, prefix = _build.build_oracle(), "mo_"
    elif kind == "reference":
        path, prefix = _build.build_reference(), "ref_"
        if path is None or not Path(path).exists():
            raise HostError("reference kernels were not built (oracle/_ref/libref_kernels.so missing)")
    else:
        raise ValueError(f"unknown kernel library {kind!r}")
    lib = C.CDLL(str(path))
    for name, (rank, kinds) in SIGNATURES.items():
        fn = getattr(lib, prefix + name)
        fn.restype = None
        fn.argtypes = [C.c_size_t] * rank + [_CTYPE[k] for k in kinds]
    return lib, prefix


@dataclass(frozen=True)
class HostDevice:
    name: str = "host"
    kind: str = "cpu"
    memory_bytes: int = 1 << 40
    max_allocation_bytes: int = 1 << 40

    def to_dict(self):
        return dict(vars(self))


class HostTensor:
    """Float32 buffer with the reference Tensor attributes (shape, size, handle)."""

    def __init__(self, backend, shape):
        self.backend, self.shape = backend, tuple(shape)
        self.size = math.prod(self.shape)
        self.data = np.zeros(self.size, dtype=np.float32)

    @property
    def handle(self):
        return self.data.ctypes.data


class HostBackend:
    """Reference backend surface evaluated on host cores (see module docstring)."""

    def __init__(self, kernels: str = "oracle", max_allocation_bytes: int = 1 << 40):
        self.lib, self.prefix = load_kernels(kernels)
        self.kernels = kernels
        self.device = HostDevice(name=f"host-{kernels}", max_allocation_bytes=max_allocation_bytes)
        self.uploads = []          # optional recording hook (golden generation): True records
                                   # every upload, a predicate only the arrays it accepts
        self.record_uploads = False

    # buffers -----------------------------------------------------------------
    def empty(self, shape):
        shape = tuple(shape)
        if not shape or any(not isinstance(n, int) or n <= 0 for n in shape):
            raise ValueError(f"invalid tensor shape: {shape}")
        if math.prod(shape) * 4 > self.device.max_allocation_bytes:
            raise HostError("buffer above the device allocation limit")
        return HostTensor(self, shape)

    def upload(self, array):
        array = np.ascontiguousarray(array, dtype=np.float32)
        out = self.empty(array.shape)
        out.data[:] = array.reshape(-1)
        if self.record_uploads and (self.record_uploads is True or self.record_uploads(array)):
            self.uploads.append(array.copy())
        return out

    def read(self, tensor):
        self._owns(tensor)
        return tensor.data.reshape(tensor.shape).copy()

    def _owns(self, *tensors):
        if any(t.backend is not self for t in tensors):
            raise ValueError("Tensors belong to different backends")

    def copy(self, source, target, *, source_offset=0, target_offset=0, count=None):
        self._owns(source, target)
        count = source.size - source_offset if count is None else count
        if (min(source_offset, target_offset, count) < 0 or source_offset + count > source.size
                or target_offset + count > target.size):
            raise ValueError("tensor copy is out of bounds")
        if count:
            target.data[target_offset:target_offset + count] = \
                source.data[source_offset:source_offset + count]

    # dispatch ------------------------------------------------------------------
    def run(self, name, shape, *args):
        if name not in SIGNATURES:
            raise HostError(f"unknown kernel {name}")
        rank, kinds = SIGNATURES[name]
        if len(shape) != rank or len(args) != len(kinds):
            raise ValueError(f"{name}: bad launch shape or argument count")
        values = []
        for arg in args:
            if isinstance(arg, HostTensor):
                self._owns(arg)
                values.append(C.c_void_p(arg.handle))
            elif isinstance(arg, (float, np.floating)):
                values.append(C.c_float(arg))
            elif isinstance(arg, (int, np.integer)) and -(2 ** 31) <= arg < 2 ** 31:
                values.append(C.c_int(arg))
            else:
                raise ValueError(f"unsupported kernel argument: {arg}")
        for value, kind in zip(values, kinds):
            if (kind == _P) != isinstance(value, C.c_void_p):
                raise ValueError(f"{name}: argument kind mismatch")
        getattr(self.lib, self.prefix + name)(*shape, *values)

    # op helpers (same launch geometry as opencl.py:241-300) ---------------------
    def linear(self, x, weight):
        if len(x.shape) != 2 or len(weight.shape) != 2 or x.shape[1] != weight.shape[1]:
            raise ValueError("linear needs x[rows,in] and weight[out,in]")
        rows, inner = x.shape
        out = self.empty((rows, weight.shape[0]))
        self.run("linear", (weight.shape[0], rows), x, weight, out, rows, weight.shape[0], inner)
        return out

    def norm(self, x, weight, width, eps):
        if x.size % width or (weight is not None and weight.shape != (width,)):
            raise ValueError("RMSNorm shape mismatch")
        out = self.empty(x.shape)
        self.run("rms", (x.size // width,), x, weight if weight is not None else x, out,
                 x.size // width, width, float(eps), int(weight is not None))
        return out

    def rotate(self, x, frequencies, positions, heads, dim, split_half=False):
        if x.shape != (positions.size, heads * dim):
            raise ValueError("RoPE shape mismatch")
        out = self.empty(x.shape)
        self.run("rope", (x.size // 2,), x, frequencies, positions, out, positions.size,
                 heads, dim, int(split_half))
        return out

    def add(self, x, y, scale=1.0):
        if x.shape != y.shape:
            raise ValueError("residual shapes differ")
        out = self.empty(x.shape)
        self.run("axpy", (x.size,), x, y, out, x.size, float(scale))
        return out

    def swiglu(self, gate, up):
        if gate.shape != up.shape:
            raise ValueError("SwiGLU shapes differ")
        out = self.empty(gate.shape)
        self.run("swiglu", (gate.size,), gate, up, out, gate.size)
        return out

    def softmax(self, x):
        out = self.empty(x.shape)
        self.run("softmax", (x.shape[0],), x, out, *x.shape)
        return out

    def attention(self, query, keys, values, *, heads, kv_heads, dim, start, length,
                  extra_keys=None, extra_values=None, extra_length=0):
        scores = self.empty((heads, length + extra_length))
        self.run("scores", (length + extra_length, heads), query, keys,
                 extra_keys if extra_keys is not None else keys, scores,
                 heads, kv_heads, dim, keys.shape[0], start, length, extra_length)
        return self.mix(self.softmax(scores), values, heads, kv_heads, dim, start, length,
                        extra_values, extra_length)

    def mix(self, probs, values, heads, kv_heads, dim, start, length,
            extra_values=None, extra_length=0):
        out = self.empty((1, heads * dim))
        self.run("mix", (heads * dim,), probs, values,
                 extra_values if extra_values is not None else values, out,
                 heads, kv_heads, dim, values.shape[0], start, length, extra_length)
        return out

    def finish(self):
        return None
