// Attention (scores -> softmax -> mix) that allocates no device memory.
//
// Who needs this: code that must not call cudaMalloc while it runs — a host
// framework that owns all device memory through its own pool or arena, or a
// caller in a section where an allocation could synchronize the device or
// fail under memory pressure.  The regular path (CUDABackend.attention, or
// mr_op_scores + mr_op_softmax + mr_op_mix) needs a [heads x (length +
// extra_length)] score buffer per call; this variant keeps that buffer in one
// file-scope device array instead.
//
// Limits and sharing rules:
//   * the array holds kStaticScratchFloats floats (4 MiB) and is resident on
//     every GPU that loads this library until the process exits;
//   * heads * (length + extra_length) must fit in it, otherwise the call
//     fails with MR_ERR_ARGUMENT and does nothing;
//   * every call on a device uses the same array; the array keeps whatever
//     the last call left there.  Each call writes every score it later reads,
//     so nothing has to start at zero, but calls that overlap on the GPU (two
//     streams, or two host threads) race on the array and must be serialised
//     by the caller;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make that
//     first call before any stream capture.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kStaticScratchFloats = size_t(1) << 20;
constexpr int kMaxDevices = 64;
constexpr int kThreads = 256;

// Host code must never hand this symbol to a kernel: on the host it names a
// stand-in, not device memory.  Kernels receive the address looked up below.
static __device__ __align__(256) float g_attention_scratch[kStaticScratchFloats];

std::mutex g_scratch_lock;
float *g_scratch_address[kMaxDevices] = {};

int scratch_address(int device, float **out) {
    std::lock_guard<std::mutex> guard(g_scratch_lock);
    if (!g_scratch_address[device]) {
        void *address = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&address, g_attention_scratch);
        if (err != cudaSuccess) return mr::cuda_error(err, "cudaGetSymbolAddress(attention scratch)");
        g_scratch_address[device] = static_cast<float *>(address);
    }
    *out = g_scratch_address[device];
    return MR_OK;
}

__device__ float block_max(float v, float *shared) {
    for (int offset = 16; offset > 0; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) shared[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < static_cast<int>(blockDim.x >> 5) ? shared[lane] : -INFINITY;
        for (int offset = 16; offset > 0; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
        if (lane == 0) shared[0] = v;
    }
    __syncthreads();
    v = shared[0];
    __syncthreads();
    return v;
}

// Row of logical key t: ring rows (start + t) mod capacity for t < length (in
// 64-bit arithmetic, so a start near INT_MAX cannot wrap), then extra rows.
// capacity is only used for ring rows, so length 0 with capacity 0 is valid.
__device__ __forceinline__ size_t logical_row(int t, int start, int length, int capacity) {
    return t < length ? (static_cast<size_t>(start) + static_cast<size_t>(t)) % static_cast<size_t>(capacity)
                      : static_cast<size_t>(t - length);
}

// One block per query head; scores of head h live in scores[h * total ...].
__global__ void k_attention_static(const float *q, const float *keys, const float *values, const float *extra_keys,
                                   const float *extra_values, float *out, float *scores, int heads, int kv_heads,
                                   int dim, int capacity, int start, int length, int extra_length) {
    __shared__ float shared[32];
    const int h = blockIdx.x, total = length + extra_length, kh = h / (heads / kv_heads);
    float *s = scores + static_cast<size_t>(h) * total;
    const float sqrt_dim = __fsqrt_rn(static_cast<float>(dim));
    for (int t = threadIdx.x; t < total; t += blockDim.x) {
        const size_t row = logical_row(t, start, length, capacity);
        const float *k = (t < length ? keys : extra_keys) + (row * kv_heads + kh) * dim;
        float dot = 0.f;
        for (int j = 0; j < dim; ++j) dot = __fadd_rn(dot, __fmul_rn(q[h * dim + j], k[j]));
        s[t] = __fdiv_rn(dot, sqrt_dim);
    }
    __syncthreads();
    // softmax (kernels.cl:75-84): the maximum in any order (fmax is exact), the
    // exponentials in parallel, their sum by one thread in row order, as the
    // reference's work item sums it
    float m = -INFINITY;
    for (int t = threadIdx.x; t < total; t += blockDim.x) m = fmaxf(m, s[t]);
    m = block_max(m, shared);
    for (int t = threadIdx.x; t < total; t += blockDim.x) s[t] = expf(__fsub_rn(s[t], m));
    __syncthreads();
    if (threadIdx.x == 0) {
        float denom = 0.f;
        for (int t = 0; t < total; ++t) denom = __fadd_rn(denom, s[t]);
        shared[0] = denom;
    }
    __syncthreads();
    const float denom = shared[0];
    for (int t = threadIdx.x; t < total; t += blockDim.x) s[t] = __fdiv_rn(s[t], denom);
    __syncthreads();
    for (int j = threadIdx.x; j < dim; j += blockDim.x) {
        float acc = 0.f;
        for (int t = 0; t < total; ++t) {
            const size_t row = logical_row(t, start, length, capacity);
            const float *v = (t < length ? values : extra_values) + (row * kv_heads + kh) * dim;
            acc = __fadd_rn(acc, __fmul_rn(s[t], v[j]));
        }
        out[static_cast<size_t>(h) * dim + j] = acc;
    }
}

}  // namespace

extern "C" int mr_attention_static_scratch(mr_context *ctx, const float *q, const float *keys, const float *values,
                                           const float *extra_keys, const float *extra_values, float *out, int heads,
                                           int kv_heads, int dim, int capacity, int start, int length,
                                           int extra_length) {
    MR_REQUIRE(ctx, "ctx is NULL");
    MR_REQUIRE(ctx->device >= 0 && ctx->device < kMaxDevices, "device %d out of range", ctx->device);
    MR_REQUIRE(q && out, "q and out must be device pointers");
    MR_REQUIRE(heads > 0 && kv_heads > 0 && heads % kv_heads == 0, "heads must be a positive multiple of kv_heads");
    MR_REQUIRE(dim > 0 && length >= 0 && extra_length >= 0 && length + extra_length > 0 && start >= 0,
               "invalid attention geometry");
    MR_REQUIRE(length == 0 || (keys && values && capacity > 0), "ring keys/values and a positive capacity are needed");
    MR_REQUIRE(extra_length == 0 || (extra_keys && extra_values), "extra keys/values are needed");
    const size_t need = static_cast<size_t>(heads) * static_cast<size_t>(length + extra_length);
    MR_REQUIRE(need <= kStaticScratchFloats,
               "attention needs %zu floats of scratch (heads x (length + extra_length)); the static scratch holds %zu",
               need, kStaticScratchFloats);
    MR_CUDA_TRY(cudaSetDevice(ctx->device));
    float *scratch = nullptr;
    int rc = scratch_address(ctx->device, &scratch);
    if (rc) return rc;
    k_attention_static<<<heads, kThreads, 0, ctx->stream>>>(q, keys, values, extra_keys, extra_values, out, scratch,
                                                           heads, kv_heads, dim, capacity, start, length,
                                                           extra_length);
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}
