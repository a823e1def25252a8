// Shared host/device helpers of libmiracle_cuda.so (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/miracle_cuda.h"

// ---- host-side error reporting ------------------------------------------------
namespace mr {

int set_error(int code, const char *fmt, ...);
int cuda_error(cudaError_t err, const char *what);

}  // namespace mr

#define MR_CUDA_TRY(call)                                                       \
    do {                                                                        \
        cudaError_t _e = (call);                                                \
        if (_e != cudaSuccess) return mr::cuda_error(_e, #call);                \
    } while (0)

#define MR_REQUIRE(cond, ...)                                                   \
    do {                                                                        \
        if (!(cond)) return mr::set_error(MR_ERR_ARGUMENT, __VA_ARGS__);        \
    } while (0)

// A context is shared by its creator and by every buffer and model made on
// it; each holds one reference and the last release destroys the stream.  So
// the handles can be released in any order (a garbage-collected host
// language finalises them in no fixed order at exit).
struct mr_context {
    int device = 0;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    size_t max_allocation = 0;
    std::atomic<int> refs{1};
};

namespace mr {
inline void context_retain(mr_context *ctx) { ctx->refs.fetch_add(1, std::memory_order_relaxed); }
inline void context_release(mr_context *ctx) {
    if (ctx->refs.fetch_sub(1, std::memory_order_acq_rel) != 1) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
}
}  // namespace mr

struct mr_buffer {
    mr_context *ctx = nullptr;
    float *ptr = nullptr;
    size_t count = 0;
};

// ---- device helpers --------------------------------------------------------------
namespace mr {

// Stored weight element -> float32, exactly as the reference widens on the host:
// BF16 bits << 16 (weights.py:70), F16 via IEEE half->float (exact).
__device__ __forceinline__ float widen_bf16(uint16_t bits) {
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}
__device__ __forceinline__ float widen_f16(uint16_t bits) {
    return __half2float(__ushort_as_half(bits));
}
__device__ __forceinline__ float load_weight(const void *base, int dtype, size_t index) {
    if (dtype == MR_DTYPE_F32) return static_cast<const float *>(base)[index];
    uint16_t bits = static_cast<const uint16_t *>(base)[index];
    return dtype == MR_DTYPE_BF16 ? widen_bf16(bits) : widen_f16(bits);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
    return v;
}

// Nanoseconds from the global timer (bounded waits).
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Bulk L2 prefetch of [ptr, ptr+bytes) (no completion to wait for).  Address
// rounded down and end rounded up to 16 bytes, as cp.async.bulk requires;
// every tensor allocation is padded to 256 bytes so the rounding stays inside.
__device__ __forceinline__ void prefetch_l2(const void *ptr, size_t bytes) {
    uintptr_t begin = reinterpret_cast<uintptr_t>(ptr) & ~uintptr_t(15);
    uintptr_t end = (reinterpret_cast<uintptr_t>(ptr) + bytes + 15) & ~uintptr_t(15);
    const uintptr_t chunk = 1u << 20;  // keep each request well below the size limit
    for (uintptr_t a = begin; a < end; a += chunk) {
        uint32_t n = static_cast<uint32_t>((end - a) < chunk ? (end - a) : chunk);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
    }
}

// Argmax key: larger float -> larger key, ties -> lower index wins under max.
__device__ __forceinline__ unsigned long long argmax_key(float v, int index) {
    if (v == 0.0f) v = 0.0f;  // -0 == +0 for numpy.argmax
    uint32_t bits = __float_as_uint(v);
    uint32_t ordered = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    return (static_cast<unsigned long long>(ordered) << 32) |
           static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(index));
}
__device__ __forceinline__ int argmax_index(unsigned long long key) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
}

}  // namespace mr
