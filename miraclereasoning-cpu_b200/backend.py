"""``CUDABackend``: the reference backend's method surface on a B200.

Drop-in for ``OpenCLBackend`` (miracle_reasoning/opencl.py:129-303): the same
``empty/upload/read/copy/run/linear/norm/rotate/add/swiglu/softmax/attention/
mix/finish`` methods with the same argument meaning, shapes and error
behaviour, and a ``device`` with ``max_allocation_bytes`` and ``to_dict()``.
Tensors are float32 device buffers owned by the C library; ``run(name, ...)``
dispatches to the kernel's ``mr_op_*`` entry point.  There is no host fallback:
a missing library or device raises ``CUDAError``.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np

from . import _native
from ._native import CUDAError, call

# kernel name -> (NDRange rank, argument kinds) in kernels.cl order
_KERNELS = {
    "linear": (2, "pppiii"), "rms": (1, "pppiifi"), "rope": (1, "ppppiiii"), "swiglu": (1, "pppi"),
    "axpy": (1, "pppif"), "scores": (2, "ppppiiiiiii"), "softmax": (1, "ppii"),
    "latent_mask": (2, "ppiiii"), "mix": (1, "ppppiiiiiii"), "pool_scores": (2, "pppiii"),
    "pool_mix": (2, "ppppiiii"), "merge_rows": (1, "ppiff"), "block_means": (2, "ppiii"),
}
_KIND_NAMES = {"p": "a tensor", "i": "an int", "f": "a float"}


@dataclass(frozen=True)
class Device:
    ordinal: int
    name: str
    kind: str
    memory_bytes: int
    max_allocation_bytes: int
    sm_count: int
    compute_capability: str

    def to_dict(self):
        return dict(vars(self))


def list_devices():
    """CUDA devices visible to this process ([] when there is none)."""
    lib = _native.library()
    count = C.c_int()
    _native.check(lib.mr_device_count(C.byref(count)), "mr_device_count")
    devices = []
    for i in range(count.value):
        info = _native.DeviceInfo()
        _native.check(lib.mr_device_query(i, C.byref(info)), "mr_device_query")
        devices.append(Device(i, info.name.decode(), "gpu", int(info.memory_bytes),
                              int(info.max_allocation_bytes), info.sm_count, f"{info.cc_major}.{info.cc_minor}"))
    return devices


class Tensor:
    """float32 device buffer (reference Tensor: shape, size, handle; freed on __del__)."""

    def __init__(self, backend, handle, shape):
        self.backend, self.handle, self.shape = backend, handle, tuple(shape)
        self.size = math.prod(self.shape)

    def __del__(self):
        handle = getattr(self, "handle", None)
        if handle and _native._lib is not None:
            _native._lib.mr_buffer_free(handle)
            self.handle = None


class CUDABackend:
    """Float32 execution on one B200 (one context = one device + one stream).

    An instance must be used by a single thread at a time, as the reference
    backend requires.
    """

    def __init__(self, *, device_index=0, platform_index=None, device_type="gpu"):
        if device_type not in ("gpu", "cuda"):
            raise ValueError("CUDABackend executes on a CUDA GPU; device_type must be 'gpu'")
        devices = list_devices()
        if not 0 <= device_index < len(devices):
            raise CUDAError(f"No CUDA device {device_index} (found {len(devices)}); no automatic CPU fallback.")
        self.device = devices[device_index]
        handle = C.c_void_p()
        call("mr_context_create", device_index, C.byref(handle))
        self.context = handle

    def __del__(self):
        ctx = getattr(self, "context", None)
        if ctx and _native._lib is not None:
            _native._lib.mr_context_destroy(ctx)
            self.context = None

    # buffers (opencl.py:178-217) -------------------------------------------------
    def empty(self, shape):
        shape = tuple(shape)
        if not shape or any(not isinstance(n, int) or n <= 0 for n in shape):
            raise ValueError(f"invalid tensor shape: {shape}")
        size = math.prod(shape) * 4
        if size > self.device.max_allocation_bytes:
            raise CUDAError(f"Buffer needs {size:,} bytes, above device allocation limit "
                            f"{self.device.max_allocation_bytes:,}; reduce context or weight tile size")
        handle = C.c_void_p()
        call("mr_buffer_alloc", self.context, math.prod(shape), C.byref(handle))
        return Tensor(self, handle.value, shape)

    def upload(self, array):
        array = np.ascontiguousarray(array, dtype=np.float32)
        out = self.empty(array.shape)
        call("mr_buffer_upload", out.handle, 0, array.ctypes.data, array.size)
        return out

    def read(self, tensor):
        self._owns(tensor)
        out = np.empty(tensor.shape, dtype=np.float32)
        call("mr_buffer_download", tensor.handle, 0, out.ctypes.data, out.size)
        return out

    def _owns(self, *tensors):
        if any(t.backend is not self for t in tensors):
            raise ValueError("Tensors belong to different CUDA contexts")

    def copy(self, source, target, *, source_offset=0, target_offset=0, count=None):
        self._owns(source, target)
        count = source.size - source_offset if count is None else count
        if (min(source_offset, target_offset, count) < 0 or source_offset + count > source.size
                or target_offset + count > target.size):
            raise ValueError("tensor copy is out of bounds")
        if count:
            call("mr_buffer_copy", source.handle, target.handle, source_offset, target_offset, count)

    # dispatch (opencl.py:219-239) -------------------------------------------------
    def run(self, name, shape, *args):
        if name not in _KERNELS:
            raise CUDAError(f"create kernel {name} failed (no such kernel)")
        rank, kinds = _KERNELS[name]
        shape = tuple(int(s) for s in shape)
        if len(shape) != rank or len(args) != len(kinds):
            raise ValueError(f"{name}: NDRange rank or argument count mismatch")
        values = []
        for index, (arg, kind) in enumerate(zip(args, kinds)):
            if isinstance(arg, Tensor):
                self._owns(arg)
                value = C.c_void_p(arg.handle)
            elif isinstance(arg, (float, np.floating)):
                value = C.c_float(arg)
            elif isinstance(arg, (int, np.integer)) and -(2 ** 31) <= arg < 2 ** 31:
                value = C.c_int(arg)
            else:
                raise ValueError(f"unsupported kernel argument: {arg}")
            expected = {"p": C.c_void_p, "i": C.c_int, "f": C.c_float}[kind]
            if type(value) is not expected:
                if kind == "f" and isinstance(value, C.c_int):
                    value = C.c_float(value.value)
                else:
                    raise ValueError(f"{name}: argument {index} must be {_KIND_NAMES[kind]}")
            values.append(value)
        call(f"mr_op_{name}", self.context, *shape, *values)

    # op helpers, same launch geometry as opencl.py:241-300 ------------------------
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
        self.run("rope", (x.size // 2,), x, frequencies, positions, out, positions.size, heads, dim,
                 int(split_half))
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

    def mix(self, probs, values, heads, kv_heads, dim, start, length, extra_values=None, extra_length=0):
        out = self.empty((1, heads * dim))
        self.run("mix", (heads * dim,), probs, values,
                 extra_values if extra_values is not None else values, out,
                 heads, kv_heads, dim, values.shape[0], start, length, extra_length)
        return out

    def finish(self):
        call("mr_context_finish", self.context)
