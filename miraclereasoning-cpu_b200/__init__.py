"""B200-native engine for the MiracleReasoning token loop.

A drop-in for the reference package's public surface
(miracle_reasoning/__init__.py): ``ModelConfig``, ``MiracleModel`` and a
``CUDABackend`` that replaces ``OpenCLBackend``.  All device work goes through
the C-ABI library ``libmiracle_cuda.so`` (declared in include/miracle_cuda.h)
via ctypes; nothing here falls back to the CPU.
"""
from . import config, weights
from .config import FAMILIES, ModelConfig

__all__ = ["FAMILIES", "ModelConfig", "MiracleModel", "CUDABackend", "CUDAError", "list_devices"]


def __getattr__(name):
    # The backend and model import the native library lazily so that the
    # host-only parts (config, weights) stay importable on machines without it.
    if name in ("CUDABackend", "CUDAError", "list_devices", "Tensor"):
        from . import backend
        return getattr(backend, name)
    if name == "MiracleModel":
        from .model import MiracleModel
        return MiracleModel
    raise AttributeError(name)
