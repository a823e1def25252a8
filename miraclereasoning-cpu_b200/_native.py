"""ctypes binding of libmiracle_cuda.so (include/miracle_cuda.h).

The library is built in-tree by ``build.py`` and loaded from next to this file
(or from ``MIRACLE_CUDA_LIBRARY``).  There is no fallback: if the library is
missing or the machine has no CUDA device, the calls raise ``CUDAError``.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIBRARY_PATH = Path(os.environ.get("MIRACLE_CUDA_LIBRARY", Path(__file__).resolve().parent / "libmiracle_cuda.so"))

MR_OK, MR_ERR_ARGUMENT, MR_ERR_CUDA, MR_ERR_STATE, MR_ERR_TIMEOUT, MR_ERR_NOMEM = range(6)
FAMILY_CODES = {"flashnano-1.5": 0, "flashnano-1.6": 1, "flashnano-1.7": 2, "flashlite-2.0": 3,
                "flashlighting-2.0": 4, "heavy-medium-2.0": 5}


class CUDAError(RuntimeError):
    """A failed call into the CUDA engine (counterpart of OpenCLError)."""

    def __init__(self, message, code=MR_ERR_CUDA):
        super().__init__(message)
        self.code = code


class DeviceInfo(C.Structure):
    _fields_ = [("ordinal", C.c_int), ("sm_count", C.c_int), ("cc_major", C.c_int), ("cc_minor", C.c_int),
                ("memory_bytes", C.c_uint64), ("max_allocation_bytes", C.c_uint64), ("name", C.c_char * 256)]


class ModelConfigC(C.Structure):
    """mr_model_config: 25 int and 5 float fields, in header order."""
    _fields_ = [(name, C.c_int) for name in (
        "family", "vocab_size", "hidden_size", "layers", "query_heads", "kv_heads", "head_dim", "ffn_dim",
        "context_length", "window", "tie_embeddings", "qk_norm", "split_half_rope")] + \
        [(name, C.c_float) for name in ("norm_eps", "residual_scale", "cbr_norm_eps")] + \
        [(name, C.c_int) for name in (
            "latent_dim", "memory_slots", "cbr_chunk_size", "cbr_slots", "inner_loop_steps",
            "routed_experts", "router_groups", "router_top_k_min", "router_top_k_max", "shared_experts",
            "block_size", "global_slots")] + \
        [("router_temperature", C.c_float), ("alibi_slope", C.c_float)]


class LayerState(C.Structure):
    _fields_ = [(name, C.c_int) for name in ("present", "ring_count", "ring_capacity", "ring_length",
                                             "ring_start", "relay_count", "latent_rows", "memory_size")]


_P, _SZ, _I, _F = C.c_void_p, C.c_size_t, C.c_int, C.c_float
_IP, _FP = C.POINTER(C.c_int), C.POINTER(C.c_float)
SIGNATURES = {
    "mr_last_error": (C.c_char_p, []),
    "mr_abi_version": (_I, []),
    "mr_device_count": (_I, [_IP]),
    "mr_device_query": (_I, [_I, C.POINTER(DeviceInfo)]),
    "mr_context_create": (_I, [_I, C.POINTER(_P)]),
    "mr_context_destroy": (_I, [_P]),
    "mr_context_finish": (_I, [_P]),
    "mr_buffer_alloc": (_I, [_P, _SZ, C.POINTER(_P)]),
    "mr_buffer_free": (_I, [_P]),
    "mr_buffer_count": (_I, [_P, C.POINTER(_SZ)]),
    "mr_buffer_upload": (_I, [_P, _SZ, _P, _SZ]),
    "mr_buffer_download": (_I, [_P, _SZ, _P, _SZ]),
    "mr_buffer_copy": (_I, [_P, _P, _SZ, _SZ, _SZ]),
    "mr_op_linear": (_I, [_P, _SZ, _SZ, _P, _P, _P, _I, _I, _I]),
    "mr_op_rms": (_I, [_P, _SZ, _P, _P, _P, _I, _I, _F, _I]),
    "mr_op_rope": (_I, [_P, _SZ, _P, _P, _P, _P, _I, _I, _I, _I]),
    "mr_op_swiglu": (_I, [_P, _SZ, _P, _P, _P, _I]),
    "mr_op_axpy": (_I, [_P, _SZ, _P, _P, _P, _I, _F]),
    "mr_op_scores": (_I, [_P, _SZ, _SZ, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I]),
    "mr_op_softmax": (_I, [_P, _SZ, _P, _P, _I, _I]),
    "mr_op_latent_mask": (_I, [_P, _SZ, _SZ, _P, _P, _I, _I, _I, _I]),
    "mr_op_mix": (_I, [_P, _SZ, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I]),
    "mr_op_pool_scores": (_I, [_P, _SZ, _SZ, _P, _P, _P, _I, _I, _I]),
    "mr_op_pool_mix": (_I, [_P, _SZ, _SZ, _P, _P, _P, _P, _I, _I, _I, _I]),
    "mr_op_merge_rows": (_I, [_P, _SZ, _P, _P, _I, _F, _F]),
    "mr_op_block_means": (_I, [_P, _SZ, _SZ, _P, _P, _I, _I, _I]),
    "mr_model_create": (_I, [_P, C.POINTER(ModelConfigC), _IP, _IP, _FP, C.POINTER(_P)]),
    "mr_model_destroy": (_I, [_P]),
    "mr_model_load_tensor": (_I, [_P, C.c_char_p, _I, _I, C.POINTER(C.c_int64), _P]),
    "mr_model_fill_synthetic": (_I, [_P, C.c_char_p, _I, _I, C.POINTER(C.c_int64), C.c_uint64, _I, _F, _F]),
    "mr_model_finalize": (_I, [_P]),
    "mr_model_reset": (_I, [_P]),
    "mr_model_set_batched_prefill": (_I, [_P, _I, _IP]),
    "mr_model_set_tensor_parallel": (_I, [_P, _I, _I]),
    "mr_model_tp_handle": (_I, [_P, _P, _SZ]),
    "mr_model_tp_connect": (_I, [_P, _P, _SZ]),
    "mr_model_position": (_I, [_P, _IP]),
    "mr_model_weight_bytes": (_I, [_P, C.POINTER(C.c_uint64)]),
    "mr_model_step": (_I, [_P, _I, _FP, _IP]),
    "mr_model_prefill": (_I, [_P, _IP, _I, _I, _FP]),
    "mr_model_generate_greedy": (_I, [_P, _IP, _I, _I, _I, _IP, _IP, _IP]),
    "mr_model_generate_sampled": (_I, [_P, _IP, _I, _I, _I, C.c_double, _I, C.c_double, C.POINTER(C.c_uint64), _IP,
                                      _IP, _IP]),
    "mr_model_layer_state": (_I, [_P, _I, _I, C.POINTER(LayerState)]),
    "mr_model_latent_positions": (_I, [_P, _I, _IP, _I, _IP]),
    "mr_model_latent_counts": (_I, [_P, _I, _FP, _I, _IP]),
    "mr_model_last_topk": (_I, [_P, _I, _I, _IP, _I]),
    "mr_model_last_experts": (_I, [_P, _I, _I, _IP, _FP, _I]),
    "mr_model_set_log1p_table": (_I, [_P, _FP, _I]),
    "mr_model_bench_decode": (_I, [_P, _I, _I, _FP]),
    "mr_model_trace_decode": (_I, [_P, _I, C.POINTER(C.c_uint64), _I, _IP, _IP]),
    "mr_attention_static_scratch": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I]),
    "mr_model_set_wait_limit": (_I, [_P, C.c_uint64]),
    "mr_model_load_file": (_I, [_P, C.c_char_p, _I, _I, C.POINTER(C.c_int64), C.c_char_p, C.c_uint64]),
    "mr_model_inject_fault": (_I, [_P, _I]),
    "mr_model_linear": (_I, [_P, C.c_char_p, _P, _I, _P]),
    "mr_model_tensor_rows": (_I, [_P, C.c_char_p, C.c_int64, C.c_int64, _P]),
    "mr_model_tensor_download": (_I, [_P, C.c_char_p, _FP, _SZ]),
}

_lib = None


def library():
    """Load (once) and return the ctypes library; raises CUDAError if it is missing."""
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise CUDAError(f"{LIBRARY_PATH} is missing: build it with "
                            f"'python miraclereasoning-cpu_b200/build.py' (no CPU fallback exists)")
        lib = C.CDLL(str(LIBRARY_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = restype, argtypes
        _lib = lib
    return _lib


def check(code, what=""):
    if code != MR_OK:
        message = library().mr_last_error().decode("utf-8", "replace")
        raise CUDAError(f"{what}: {message}" if what else message, code)


def call(name, *args):
    check(getattr(library(), name)(*args), name)
