// Heavy Medium 2.0 token step on the device (miracle_reasoning/model.py:
// 192-285): latent sparse attention with top-k global blocks, then the
// adaptive mixture of experts, two inner loops per layer, with every discrete
// decision taken on the GPU.  One call runs a token end to end from the host
// with kernel launches only: no host round trip inside a step.
//
// Per (layer, inner loop):
//   1-2. h = RMSNorm(x, a_norm) (while staging the input);
//      q = W_q h, latent = W_latent h                            k_gemv (two segments)
//   3. kv = W_kv_up latent                                       k_gemv
//   4. q = RoPE(RMSNorm_noaffine(q)); k = RoPE(RMSNorm_noaffine(kv[:w]));
//      append k, v = kv[w:] to the loop's ring                   k_heads_norm_rope
//   5. mean key / value of the newest block (older blocks' means
//      never change once full)                                   k_block_mean_last
//   6. scores over the local window and every block mean        k_sparse_scores
//   7. block columns minus the distance penalty, stable top
//      `global_slots` per head, the rest masked (model.py:219-225) k_block_topk
//   8. softmax + value mix over window rows and kept blocks     k_sparse_attend
//   9. x += s * W_o attended                                     k_gemv (residual)
//  10. f = RMSNorm(x, f_norm) (while staging); router logits    k_gemv
//  11. routing (model.py:235-250): biases, temperature, softmax,
//      stable top-k, confidence / entropy -> active count,
//      renormalised weights                                      k_route
//  12. the chosen experts and the shared experts, batched:
//      SwiGLU(gate, up), then down                               k_expert_gate_up, k_expert_down
//  13. result = sum in rank order, shared experts at
//      residual_scale / S; x += s * result                       k_expert_combine
//
// Arithmetic: the discrete decisions follow the reference's float32
// expressions in the reference's order (block means as running sums, the
// distance penalty from a table of NumPy's own float32 log1p values supplied
// by the host, the router softmax as one running sum, NumPy's pairwise
// summation for the routing entropy and the weight renormalisation, stable
// ordering with ties to the lower index).  The projections and attention sums
// are float32 with their own summation order, so logits agree with the
// reference within the parity tolerance and decisions agree except where the
// reference's own values tie within rounding.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "heavy.cuh"
#include "prefill.cuh"
#include "tcgen05.cuh"

namespace mr {

int model_tensor(mr_model *m, const char *name, const void **ptr, int *dtype, int64_t *rows, int64_t *cols);

namespace {

constexpr int kGemvThreads = 256;  // 8 warps
constexpr int kGemvRows = 8;       // rows per block (one per warp)
constexpr int kMaxSegs = 4;
constexpr int kMaxHeavyRanks = 8;
constexpr uint64_t kHeavyWaitNs = 2000000000ull;  // 2 s: a rank that never publishes is an error, not a hang
constexpr int kStreamSmem = 227 * 1024;  // dynamic shared memory of a streaming CTA (the ring takes what is left)

__device__ __forceinline__ uint64_t global_time_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

#define FADD __fadd_rn
#define FMUL __fmul_rn

// Programmatic dependent launch: every kernel lets the next one be scheduled
// as soon as it starts (pdl_trigger), and waits for the previous one to
// complete, with its writes visible, before it reads anything an earlier
// kernel wrote or writes anything (pdl_wait).  Only loads of the weights,
// which nothing writes, come before the wait: the weight stream of a GEMV
// starts while the kernel before it finishes.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 16 bytes of weights (8 BF16 / F16 or 4 F32) dotted with the matching x.
__device__ __forceinline__ float dot16(const uint4 &w, const float *x, int dtype) {
    if (dtype == MR_DTYPE_F32) {
        const float4 a = *reinterpret_cast<const float4 *>(x);
        return __uint_as_float(w.x) * a.x + __uint_as_float(w.y) * a.y + __uint_as_float(w.z) * a.z +
               __uint_as_float(w.w) * a.w;
    }
    const float4 a = *reinterpret_cast<const float4 *>(x), b = *reinterpret_cast<const float4 *>(x + 4);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
    float lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (dtype == MR_DTYPE_BF16) {
            lo[i] = __uint_as_float(u[i] << 16);
            hi[i] = __uint_as_float(u[i] & 0xffff0000u);
        } else {
            lo[i] = __half2float(__ushort_as_half(static_cast<uint16_t>(u[i] & 0xffffu)));
            hi[i] = __half2float(__ushort_as_half(static_cast<uint16_t>(u[i] >> 16)));
        }
    }
    float s = lo[0] * a.x;
    s = fmaf(hi[0], a.y, s);
    s = fmaf(lo[1], a.z, s);
    s = fmaf(hi[1], a.w, s);
    s = fmaf(lo[2], b.x, s);
    s = fmaf(hi[2], b.y, s);
    s = fmaf(lo[3], b.z, s);
    s = fmaf(hi[3], b.w, s);
    return s;
}

// The first N 16-byte chunks per lane of up to two rows, loaded before the
// block stages its input so that the weight stream starts at once.  (Sixteen
// per lane, a whole 4096-wide BF16 row, measured no faster: the registers
// halve the resident blocks.)
constexpr int kBatch = 8;
template <int N>
struct RowBatchT {
    uint4 w0[N], w1[N];
};
__device__ __forceinline__ bool whole_chunks(int dtype, int cols) {
    return ((static_cast<size_t>(cols) * (dtype == MR_DTYPE_F32 ? 4 : 2)) & 15) == 0;
}
template <int N>
__device__ __forceinline__ void load_batch(const char *p0, const char *p1, int nv, int c0, RowBatchT<N> &b) {
#pragma unroll
    for (int u = 0; u < N; ++u) {
        const int c = c0 + 32 * u;
        b.w0[u] = c < nv ? ld_stream16(p0 + 16 * c) : make_uint4(0u, 0u, 0u, 0u);
        b.w1[u] = (p1 && c < nv) ? ld_stream16(p1 + 16 * c) : make_uint4(0u, 0u, 0u, 0u);
    }
}
template <int N>
__device__ __forceinline__ void prefetch_rows(const char *p0, const char *p1, int dtype, int cols, RowBatchT<N> &b) {
    if (whole_chunks(dtype, cols)) load_batch(p0, p1, cols / (dtype == MR_DTYPE_F32 ? 4 : 8), threadIdx.x & 31, b);
}

// One warp: dot products of up to two rows (cols elements of `dtype` at p0,
// p1; p1 NULL: one row) with x (shared memory), the first chunks already in
// `b` (prefetch_rows); every lane gets the sums.  Each lane keeps N 16-byte
// loads of a row in flight.
template <int N>
__device__ __forceinline__ void warp_dot2(const char *p0, const char *p1, int dtype, int cols, const float *x,
                                          RowBatchT<N> &b, float &y0, float &y1) {
    const int lane = threadIdx.x & 31;
    const int per = dtype == MR_DTYPE_F32 ? 4 : 8;
    float a0 = 0.f, a1 = 0.f;
    if (whole_chunks(dtype, cols)) {
        const int nv = cols / per;
        for (int c0 = lane;;) {
#pragma unroll
            for (int u = 0; u < N; ++u) {
                const int c = c0 + 32 * u;
                if (c < nv) {
                    a0 += dot16(b.w0[u], x + per * c, dtype);
                    if (p1) a1 += dot16(b.w1[u], x + per * c, dtype);
                }
            }
            c0 += 32 * N;
            if (c0 >= nv) break;
            load_batch(p0, p1, nv, c0, b);
        }
    } else {  // rows that are not whole 16-byte chunks: element by element
        for (int j = lane; j < cols; j += 32) {
            a0 = fmaf(load_weight(p0, dtype, j), x[j], a0);
            if (p1) a1 = fmaf(load_weight(p1, dtype, j), x[j], a1);
        }
    }
    y0 = warp_sum(a0);
    y1 = warp_sum(a1);
}

// Stages x (n floats) in shared memory, or RMSNorm(x) with `gain`
// (kernels.cl:19-28: (x * (1 / sqrt(mean(x^2) + eps))) * gain) when `norm`:
// every block computes the same factor from the same sums.
// The loads are 16-byte vectors issued several at a time: a loop of
// dependent scalar loads here costs more than the block's whole weight stream.
__device__ void stage_input(const float *x, int n, bool norm, const void *gain, int gain_dtype, float eps,
                            float *xs) {
    __shared__ float red[32];
    float ss = 0.f;
    const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (vec) {
#pragma unroll 4
        for (int i = 4 * threadIdx.x; i < n; i += 4 * blockDim.x) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + i));
            *reinterpret_cast<float4 *>(xs + i) = v;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
    } else {
#pragma unroll 4
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float v = x[i];
            xs[i] = v;
            ss = fmaf(v, v, ss);
        }
    }
    if (!norm) {
        __syncthreads();
        return;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += red[w];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(FADD(__fdiv_rn(total, static_cast<float>(n)), eps)));
    if (vec && gain && gain_dtype != MR_DTYPE_F32 && (reinterpret_cast<uintptr_t>(gain) & 7) == 0) {
#pragma unroll 4
        for (int i = 4 * threadIdx.x; i < n; i += 4 * blockDim.x) {  // four 16-bit gains per 8-byte load
            const uint2 g = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(gain) + i));
            const uint16_t h[4] = {static_cast<uint16_t>(g.x & 0xffffu), static_cast<uint16_t>(g.x >> 16),
                                   static_cast<uint16_t>(g.y & 0xffffu), static_cast<uint16_t>(g.y >> 16)};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float gv = gain_dtype == MR_DTYPE_BF16 ? widen_bf16(h[k]) : widen_f16(h[k]);
                xs[i + k] = FMUL(FMUL(xs[i + k], scale), gv);
            }
        }
    } else {
#pragma unroll 4
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float g = gain ? load_weight(gain, gain_dtype, i) : 1.0f;
            xs[i] = FMUL(FMUL(xs[i], scale), g);
        }
    }
    __syncthreads();
}

// Tracing probes of one launch (NULL when not tracing): [0] first CTA start,
// [1] first CTA past the dependency wait, [2] last CTA done staging its
// input, [3] last CTA done with its main loop, [4] last CTA exit.
enum ProbePoint {
    kProbeStart = 0, kProbeWaited = 1, kProbeStaged = 2, kProbeMain = 3, kProbeExit = 4,
    kProbeX5 = 5, kProbeX6 = 6, kProbeX7 = 7,  // kernel-specific, latest over CTAs
    kProbeSlots = 8
};
__device__ __forceinline__ void probe(unsigned long long *p, int point) {
    if (!p) return;
    const unsigned long long t = global_time_ns();
    if (point <= kProbeWaited) atomicMin(p + point, t);
    else atomicMax(p + point, t);
}

struct GemvSeg {
    const void *w;
    int dtype, rows, cols;
    const float *x;
    float *y;
    int residual;  // y = y + scale * (W x) (kernels.cl add), else y = W x
    float scale;
    int norm;      // the input is RMSNorm(x, gain) (computed while staging)
    const void *gain;
    int gain_dtype;
    float eps;
};
struct GemvArgs {
    GemvSeg s[kMaxSegs];
    int first[kMaxSegs + 1];  // first block of each segment
    int nseg;
};

// y = W x for up to kMaxSegs matrices; each block takes kGemvRows rows (one
// per warp) of one segment and stages that segment's input in shared memory.
__global__ void __launch_bounds__(kGemvThreads) k_gemv(GemvArgs a) {
    extern __shared__ __align__(16) float xs[];
    pdl_trigger();
    int si = 0;
    while (si + 1 < a.nseg && static_cast<int>(blockIdx.x) >= a.first[si + 1]) ++si;
    const GemvSeg &s = a.s[si];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = (blockIdx.x - a.first[si]) * kGemvRows + warp;
    const size_t row_bytes = static_cast<size_t>(s.cols) * (s.dtype == MR_DTYPE_F32 ? 4 : 2);
    const char *row = static_cast<const char *>(s.w) + static_cast<size_t>(min(r, s.rows - 1)) * row_bytes;
    RowBatchT<kBatch> b;
    if (r < s.rows) prefetch_rows(row, nullptr, s.dtype, s.cols, b);
    pdl_wait();
    stage_input(s.x, s.cols, s.norm != 0, s.gain, s.gain_dtype, s.eps, xs);
    if (r >= s.rows) return;
    float y, unused;
    warp_dot2(row, nullptr, s.dtype, s.cols, xs, b, y, unused);
    if (lane == 0) s.y[r] = s.residual ? FADD(s.y[r], FMUL(s.scale, y)) : y;
}

// x = embed[token]; the token from `dtoken` (device) when given.
__global__ void k_embed_row(const void *embed, int dtype, const int *dtoken, int token, int width, float *x) {
    pdl_trigger();
    pdl_wait();
    if (dtoken) token = *dtoken;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < width; j += gridDim.x * blockDim.x)
        x[j] = load_weight(embed, dtype, static_cast<size_t>(token) * width + j);
}

// numpy.argmax of the logits (the first maximum) into *token: the next greedy token.
__global__ void k_argmax(const float *v, int n, int *token) {
    pdl_trigger();
    pdl_wait();
    __shared__ float best_v[32];
    __shared__ int best_i[32];
    float bv = -INFINITY;
    int bi = n;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (v[i] > bv || (v[i] == bv && i < bi)) {
            bv = v[i];
            bi = i;
        }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        best_v[threadIdx.x >> 5] = bv;
        best_i[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (best_v[w] > bv || (best_v[w] == bv && best_i[w] < bi)) {
                bv = best_v[w];
                bi = best_i[w];
            }
        *token = bi < n ? bi : 0;
    }
}

// Tracing: records %globaltimer once the kernel before it has completed
// (after griddepcontrol.wait, so its writes are visible), i.e. the step's
// kernel-boundary times as the pipelined launches actually run.
__global__ void k_stamp(unsigned long long *slot) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) *slot = global_time_ns();
}

// NumPy's pairwise float32 summation (np.add.reduce over a contiguous axis):
// fewer than 8 terms in order; up to 128 in eight interleaved running sums
// combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) plus the tail in order;
// larger halves recursively (at a multiple of 8).
// NumPy's pairwise summation of float32 (identity start; eight running sums up
// to 128 values; halves above, the first a multiple of 8), without recursion:
// an explicit stack visits the halves in the same order.
__device__ float numpy_pairwise_leaf(const float *a, int n) {
    if (n < 8) {
        float res = 0.f;
        for (int i = 0; i < n; ++i) res = FADD(res, a[i]);
        return res;
    }
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
        for (int j = 0; j < 8; ++j) r[j] = FADD(r[j], a[i + j]);
    float res = FADD(FADD(FADD(r[0], r[1]), FADD(r[2], r[3])), FADD(FADD(r[4], r[5]), FADD(r[6], r[7])));
    for (; i < n; ++i) res = FADD(res, a[i]);
    return res;
}
__device__ float numpy_pairwise_sum(const float *a, int n) {
    constexpr int kDepth = 32;
    int start[kDepth], len[kDepth], phase[kDepth];
    float left[kDepth];
    int top = 0;
    start[0] = 0;
    len[0] = n;
    phase[0] = 0;
    float value = 0.f;
    while (top >= 0) {
        const int m = len[top];
        if (m <= 128) {
            value = numpy_pairwise_leaf(a + start[top], m);
            --top;
            continue;
        }
        const int n2 = m / 2 - (m / 2) % 8;
        if (phase[top] == 0) {
            phase[top] = 1;
            start[top + 1] = start[top];
            len[top + 1] = n2;
            phase[top + 1] = 0;
            ++top;
        } else if (phase[top] == 1) {
            phase[top] = 2;
            left[top] = value;
            start[top + 1] = start[top] + n2;
            len[top + 1] = m - n2;
            phase[top + 1] = 0;
            ++top;
        } else {
            value = FADD(left[top], value);
            --top;
        }
    }
    return value;
}

struct RouteArgs {
    const float *router;         // [groups + experts]: coarse logits, then fine
    const void *coarse_bias, *group_bias, *fine_bias, *expert_bias;
    int bias_dtype[4];
    int experts, groups, per_group, max_k, min_k;
    float temperature, log_experts;  // float32(max(T, 1e-4)), float32(log(E))
    int *chosen;                 // [max_k] expert ids in rank order, -1 after the active ones
    float *weights;              // [max_k]
    int *active;                 // 1
};

// model.py:233-250 for one token (at most 256 experts, one thread each):
// the element-wise steps in parallel, the running sums and the final
// arithmetic in thread 0 in the reference's order.
__device__ void route_block(const RouteArgs &a) {
    __shared__ float coarse[256], logits[256], ex[256], probs[256], terms[256];
    __shared__ int order[64];
    __shared__ float m_s, den_s;
    const int t = threadIdx.x, E = a.experts, G = a.groups, K = a.max_k;
    if (t < G)
        coarse[t] = FADD(__ldcg(a.router + t), FADD(load_weight(a.coarse_bias, a.bias_dtype[0], t),
                                           load_weight(a.group_bias, a.bias_dtype[1], t)));
    if (t < K) order[t] = -1;
    __syncthreads();
    if (t < E) {
        const float fine = FADD(__ldcg(a.router + G + t), FADD(load_weight(a.fine_bias, a.bias_dtype[2], t),
                                                     load_weight(a.expert_bias, a.bias_dtype[3], t)));
        logits[t] = __fdiv_rn(FADD(fine, coarse[min(t / a.per_group, G - 1)]), a.temperature);
    }
    __syncthreads();
    // the softmax kernel (kernels.cl:76-84): the maximum (exact in any order: warp 0),
    // then one running sum in expert order (thread 0, eight terms loaded at a time)
    if (t < 32) {
        float m = -INFINITY;
        for (int e = t; e < E; e += 32) m = fmaxf(m, logits[e]);
        m = warp_max(m);
        if (t == 0) m_s = m;
    }
    __syncthreads();
    if (t < E) ex[t] = expf(__fsub_rn(logits[t], m_s));
    __syncthreads();
    if (t == 0) {
        float den = 0.f;
        for (int e0 = 0; e0 < E; e0 += 8) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = e0 + k < E ? ex[e0 + k] : 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (e0 + k < E) den = FADD(den, v[k]);
        }
        den_s = den;
    }
    __syncthreads();
    if (t < E) probs[t] = __fdiv_rn(ex[t], den_s);
    __syncthreads();
    if (t < E) {
        // np.argsort(-probs, kind="stable")[:max_k]: rank = greater values, then equal ones before it
        const float v = probs[t];
        int rank = 0;
        for (int j = 0; j < E; ++j) rank += (probs[j] > v) || (probs[j] == v && j < t);
        if (rank < K) order[rank] = t;
        terms[t] = FMUL(v, logf(fmaxf(v, 1e-9f)));
    }
    __syncthreads();
    if (t != 0) return;
    float sel[64];
    for (int k = 0; k < K; ++k) sel[k] = order[k] >= 0 ? probs[order[k]] : 0.f;
    const float confidence = __fsub_rn(sel[0], sel[min(K - 1, 1)]);
    const float entropy = -numpy_pairwise_sum(terms, E);
    const float width = rintf(FADD(FMUL(__fsub_rn(1.0f, confidence), 2.0f),
                                   __fdiv_rn(entropy, fmaxf(a.log_experts, 1.0f))));
    const float total = FADD(static_cast<float>(a.min_k), width);
    const int active = static_cast<int>(fminf(fmaxf(total, static_cast<float>(a.min_k)), static_cast<float>(K)));
    for (int k = active; k < K; ++k) sel[k] = 0.f;
    const float norm = fmaxf(numpy_pairwise_sum(sel, K), 1e-9f);
    for (int k = 0; k < K; ++k) {
        a.chosen[k] = k < active ? order[k] : -1;
        a.weights[k] = k < active ? __fdiv_rn(sel[k], norm) : 0.f;
    }
    *a.active = active;
}

#include "heavy_attn.cuh"
#include "heavy_stream.cuh"
#include "heavy_prefill.cuh"

// The router GEMV (coarse rows, then fine rows; one row per warp, the input
// RMSNorm(x, f_norm) staged per block, k_gemv's arithmetic) and then, in the
// last block to finish, the routing of route_block (model.py:233-250).
struct RouterArgs {
    RouteArgs ra;                 // routing of the logits at ra.router
    float *logits;                // = ra.router: coarse then fine logits (groups + experts)
    const void *coarse, *fine;    // [groups, cols], [experts, cols]
    int dtype, cols, groups, experts;
    const float *x;
    const void *gain;
    int gain_dtype;
    float eps;
    unsigned long long *done;     // monotonic count of finished blocks
    unsigned long long seq;       // this launch's number (1, 2, ...)
    unsigned long long *probe;    // tracing only, else NULL
};

static_assert(kGemvThreads == stream::kConsumers, "the router stages its input with stream::stage (256 threads)");
__global__ void __launch_bounds__(kGemvThreads) k_router_route(RouterArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ int last;
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows = a.groups + a.experts, r = blockIdx.x * kGemvRows + warp;
    const size_t row_bytes = static_cast<size_t>(a.cols) * (a.dtype == MR_DTYPE_F32 ? 4 : 2);
    const int rr = min(r, rows - 1);
    const char *row = rr < a.groups ? static_cast<const char *>(a.coarse) + rr * row_bytes
                                    : static_cast<const char *>(a.fine) + (rr - a.groups) * row_bytes;
    RowBatchT<kBatch> b;
    __shared__ float red[32];
    float gains[stream::kGainRegs];
    if (threadIdx.x == 0) probe(a.probe, kProbeStart);
    if (r < rows) prefetch_rows(row, nullptr, a.dtype, a.cols, b);
    stream::load_gains(a.gain, a.gain_dtype, a.cols, gains);  // weights: before the dependency wait
    pdl_wait();
    if (threadIdx.x == 0) probe(a.probe, kProbeWaited);
    // RMSNorm(x, f_norm) as stage_input computes it (256 threads), plain layout
    stream::stage(a.x, a.cols, true, a.gain, a.gain_dtype, gains, a.eps, false, xs, red);
    __syncthreads();
    if (threadIdx.x == 0) probe(a.probe, kProbeStaged);
    if (r < rows) {
        float y, unused;
        warp_dot2(row, nullptr, a.dtype, a.cols, xs, b, y, unused);
        if (lane == 0) a.logits[r] = y;
    }
    if (threadIdx.x == 0) probe(a.probe, kProbeMain);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(a.done, 1ull) == a.seq * gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    route_block(a.ra);
    if (threadIdx.x == 0) probe(a.probe, kProbeExit);
}

struct ExpertArgs {
    const void *const *gate;  // [experts + shared] matrix pointers (routed, then shared)
    const void *const *up;
    const void *const *down;
    int dtype, ffn, hidden, experts, max_k, shared;
    const int *chosen, *active;
    const float *x;           // the residual stream; the experts read RMSNorm(x, f_norm)
    const void *norm_gain;
    int norm_dtype;
    float eps;
    float *act;               // [max_k + shared][ffn] SwiGLU activations
    float *out;               // [max_k + shared][hidden] (expert parallel: this step's buffer in the arena)
    // expert parallel: expert e runs on rank e % ranks, which stores its output
    // rows into every rank's `out` (peer[j] + out_offset), then raises its flag
    int rank, ranks;
    char *peer[kMaxHeavyRanks];    // every rank's exchange arena (this rank's included)
    size_t out_offset;             // byte offset of `out` inside an arena
    unsigned long long *flags;     // this rank's arena: one word per rank
    size_t flags_offset;
    unsigned long long tag;        // this MoE step's flag value
    int *err;                      // a bounded wait gave up
    unsigned long long wait_ns;    // how long the flag wait may last
};

// Expert id of slot `slot` (routed slots in rank order, then the shared
// experts), or -1 when the slot is not active this token or another rank runs it.
__device__ __forceinline__ int slot_expert(const ExpertArgs &a, int slot) {
    const int e = slot < a.max_k ? (slot < *a.active ? a.chosen[slot] : -1) : a.experts + (slot - a.max_k);
    return (e >= 0 && e % a.ranks == a.rank) ? e : -1;
}

// act[slot][r] = silu(gate_r . x) * (up_r . x) (kernels.cl:46-50); grid (row blocks, slots).
__global__ void __launch_bounds__(kGemvThreads) k_expert_gate_up(ExpertArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float xs[];
    const int slot = blockIdx.y, e = slot_expert(a, slot);
    if (e < 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    const size_t row_bytes = static_cast<size_t>(a.hidden) * (a.dtype == MR_DTYPE_F32 ? 4 : 2);
    const size_t off = static_cast<size_t>(min(r, a.ffn - 1)) * row_bytes;
    const char *gp = static_cast<const char *>(a.gate[e]) + off, *up = static_cast<const char *>(a.up[e]) + off;
    RowBatchT<kBatch> b;
    if (r < a.ffn) prefetch_rows(gp, up, a.dtype, a.hidden, b);
    stage_input(a.x, a.hidden, true, a.norm_gain, a.norm_dtype, a.eps, xs);
    if (r >= a.ffn) return;
    float g, u;
    warp_dot2(gp, up, a.dtype, a.hidden, xs, b, g, u);
    if (lane == 0) a.act[static_cast<size_t>(slot) * a.ffn + r] = FMUL(__fdiv_rn(g, FADD(1.0f, expf(-g))), u);
}

// out[slot][r] = down_r . act[slot]; grid (row blocks, slots).
__global__ void __launch_bounds__(kGemvThreads) k_expert_down(ExpertArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float xs[];
    const int slot = blockIdx.y, e = slot_expert(a, slot);
    if (e < 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * kGemvRows + warp;
    const size_t row_bytes = static_cast<size_t>(a.ffn) * (a.dtype == MR_DTYPE_F32 ? 4 : 2);
    const char *row = static_cast<const char *>(a.down[e]) + static_cast<size_t>(min(r, a.hidden - 1)) * row_bytes;
    RowBatchT<kBatch> b;
    if (r < a.hidden) prefetch_rows(row, nullptr, a.dtype, a.ffn, b);
    stage_input(a.act + static_cast<size_t>(slot) * a.ffn, a.ffn, false, nullptr, 0, 0.f, xs);
    if (r >= a.hidden) return;
    float y, unused;
    warp_dot2(row, nullptr, a.dtype, a.ffn, xs, b, y, unused);
    const size_t at = (static_cast<size_t>(slot) * a.hidden + r) * sizeof(float);
    if (lane == 0) {
        if (a.ranks == 1) {
            a.out[static_cast<size_t>(slot) * a.hidden + r] = y;
        } else {
            for (int j = 0; j < a.ranks; ++j) *reinterpret_cast<float *>(a.peer[j] + a.out_offset + at) = y;
        }
    }
    if (a.ranks > 1) __threadfence_system();  // the rows reach every rank before the flag (k_moe_publish)
}

// model.py:251-255 then 266: result = 0; result += w_k * expert_k (rank
// order); result += (residual_scale / S) * shared_i; x += s * result, each an
// add kernel (x + scale * y, two roundings).
// Expert parallel: after every rank's expert rows of this step are stored,
// raise this rank's flag in every rank's arena (release, system scope).
__global__ void k_moe_publish(ExpertArgs a) {
    pdl_trigger();
    pdl_wait();
    __threadfence_system();
    const int j = threadIdx.x;
    if (j < a.ranks) {
        unsigned long long *f = reinterpret_cast<unsigned long long *>(a.peer[j] + a.flags_offset) + a.rank;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(a.tag) : "memory");
    }
}

__global__ void k_expert_combine(ExpertArgs a, const float *weights, float shared_scale, float scale, float *x) {
    pdl_trigger();
    pdl_wait();
    if (a.ranks > 1) {
        // every rank's flag: its expert rows of this step are here (and it has finished
        // reading the buffer of the step two back, which this step's parity reuses)
        __shared__ int ok;
        if (threadIdx.x == 0) {
            const uint64_t start = global_time_ns();
            ok = 1;
            for (int j = 0; j < a.ranks && ok; ++j) {
                for (;;) {
                    unsigned long long v;
                    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a.flags + j) : "memory");
                    if (v >= a.tag) break;
                    if (global_time_ns() - start > a.wait_ns) {
                        atomicExch(a.err, 1);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        __syncthreads();
        if (!ok) return;
    }
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.hidden) return;
    float res = 0.f;
    const int active = *a.active;
    // eight slots' rows and weights loaded at once, then summed in rank order
    for (int k0 = 0; k0 < active; k0 += 8) {
        float v[8], w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const bool in = k0 + u < active;
            v[u] = in ? a.out[static_cast<size_t>(k0 + u) * a.hidden + r] : 0.f;
            w[u] = in ? weights[k0 + u] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (k0 + u < active) res = FADD(res, FMUL(w[u], v[u]));
    }
    for (int i0 = 0; i0 < a.shared; i0 += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            v[u] = i0 + u < a.shared ? a.out[static_cast<size_t>(a.max_k + i0 + u) * a.hidden + r] : 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (i0 + u < a.shared) res = FADD(res, FMUL(shared_scale, v[u]));
    }
    x[r] = FADD(x[r], FMUL(scale, res));
}

}  // namespace

// ---- host side -------------------------------------------------------------------
struct HeavyLayer {
    const void *a_norm, *f_norm;
    int a_norm_dt, f_norm_dt;
    GemvSeg q, latent, kv_up, o, coarse, fine;
    const void *coarse_bias, *group_bias, *fine_bias, *expert_bias;
    int bias_dt[4];
    const void **d_gate, **d_up, **d_down;  // device pointer tables [experts + shared]
    std::vector<const void *> h_gate, h_up, h_down;  // the same tables on the host
    int expert_dtype;
};

// Workspace of the batched prompt (heavy_prefill.cuh) for chunks of up to `cap`
// tokens, allocated on first use: activations of the chunk, the routed rows
// sorted by expert (up to cap * max_k), the tile table, and per layer the
// router's coarse | fine rows as one BF16 matrix and the experts' weight maps.
struct HeavyBatch {
    int cap = 0, kmax = 0, max_tiles = 0;
    bool all_logits = false, ready = false;
    std::vector<void *> buffers;     // freed on growth and with the engine
    int *ids = nullptr, *err = nullptr;
    float *x = nullptr, *qlat = nullptr, *kv = nullptr, *qh = nullptr, *sum_k = nullptr, *sum_v = nullptr,
          *rlog = nullptr, *weights = nullptr, *gu = nullptr, *rout = nullptr, *sgu = nullptr, *sout = nullptr,
          *logits = nullptr, *bstate = nullptr;
    bool window_tc = false;  // the window part of the attention on tcgen05 (head_dim 128)
    uint16_t *planes = nullptr, *gplanes = nullptr, *gsplanes = nullptr;
    uint8_t *kv_planes = nullptr;  // window_tc: the key / value tiles of every 64-key block the chunk reaches
    int *chosen = nullptr, *active = nullptr, *row_of = nullptr, *token_of = nullptr, *tiles = nullptr,
        *tile_count = nullptr, *rows = nullptr;
    // per layer, kept with the engine: router rows, expert maps (gate | up pairs, down)
    uint16_t *router_w = nullptr;
    unsigned char *maps_gu = nullptr, *maps_dn = nullptr;
};

struct HeavyEngine {
    mr_model *m = nullptr;
    cudaStream_t stream = nullptr;
    int H, KVH, d, hidden, latent, ffn, vocab, layers, loops, context, window, block, slots, experts, groups,
        per_group, max_k, min_k, shared, split_half, tied;
    float eps, residual_scale, temperature, slope, log_experts;
    const void *embed, *final_norm, *head;
    int embed_dt, final_norm_dt, head_dt;
    std::vector<HeavyLayer> L;
    // device work buffers
    float *x = nullptr, *h = nullptr, *q = nullptr, *lat = nullptr, *kv = nullptr, *attn = nullptr,
          *scores = nullptr, *router = nullptr, *act = nullptr, *eout = nullptr, *logits = nullptr,
          *inv_freq = nullptr, *log1p_table = nullptr;
    std::vector<float *> k_ring, v_ring, k_mean, v_mean;  // per (layer, loop)
    int *kept = nullptr;      // [layers][loops][H][slots]
    int *chosen = nullptr;    // [layers][loops][max_k]
    float *weights = nullptr; // [layers][loops][max_k]
    int *active = nullptr;    // [layers][loops]
    int *d_token = nullptr;   // device-resident greedy decode: the next token
    // expert parallel: the exchange arena (expert rows of two steps, one flag per
    // rank), mapped by every rank; peers[j] = rank j's arena
    int rank = 0, ranks = 1;
    char *arena = nullptr;
    size_t arena_bytes = 0, out_bytes = 0, flags_offset = 0;
    char *peers[kMaxHeavyRanks] = {};
    unsigned long long moe_tag = 0;
    int *err = nullptr;
    std::vector<void *> allocations;
    bool table_set = false;
    // the streaming / fused kernels: SM count (one streaming CTA per SM), the
    // fused attention's scratch (raw key / value rows, partial softmax per
    // unit, per-KV-head counters), the newest block's running key / value sums
    // per (layer, loop), the router's block counter, and the launch numbers the
    // monotonic counters are compared against (both zeroed by heavy_reset)
    int sm_count = 0, attn_chunks = 0;
    int smem_per_sm = 0, smem_reserved = 0;  // shared memory of an SM, and what each resident CTA costs besides
    // ring slots per stream::Mode (plain, swiglu, down): measured at 4 to 12 slots, bytes in
    // flight pay more than room for the next kernel's CTAs beside a smaller ring
    int stream_slots[3] = {12, 12, 16};
    float *attn_partial = nullptr;
    unsigned long long *counters = nullptr;  // [KVH] ready, [KVH] window units done, [1] router blocks
    std::vector<float *> k_bsum, v_bsum;
    unsigned long long attn_seq = 0, route_seq = 0;
    unsigned long long wait_ns = kHeavyWaitNs;  // bounded waits (heavy_set_wait_limit)
    bool withhold = false;                      // fault injection (heavy_inject_fault)
    bool streamable = false;                 // every projection's rows are whole 16-byte chunks
    // tracing (heavy_trace_token): one stamp after every kernel of a token step
    unsigned long long *trace = nullptr;
    int trace_n = 0, trace_cap = 0;
    unsigned long long *probes = nullptr;  // kProbeSlots per probed launch (tracing)
    int probe_n = 0, probe_cap = 0;
    // batched prompt (heavy_prefill): possible when every matrix is BF16 and the engine is alone
    bool batchable = false;
    HeavyBatch batch;
};

namespace {

int halloc(HeavyEngine &e, size_t bytes, void **out) {
    void *p = nullptr;
    MR_CUDA_TRY(cudaMalloc(&p, std::max<size_t>(bytes, 16)));
    e.allocations.push_back(p);
    *out = p;
    return MR_OK;
}
template <typename T>
int halloc_n(HeavyEngine &e, size_t n, T **out) {
    void *p = nullptr;
    int rc = halloc(e, n * sizeof(T), &p);
    *out = static_cast<T *>(p);
    return rc;
}

int tensor_of(mr_model *m, const std::string &name, const void **ptr, int *dtype, int64_t *rows, int64_t *cols) {
    return model_tensor(m, name.c_str(), ptr, dtype, rows, cols);
}

int seg_of(mr_model *m, const std::string &name, const float *x, float *y, GemvSeg &s) {
    int64_t rows = 0, cols = 0;
    s = GemvSeg{};
    if (int rc = tensor_of(m, name, &s.w, &s.dtype, &rows, &cols)) return rc;
    s.rows = static_cast<int>(rows);
    s.cols = static_cast<int>(cols);
    s.x = x;
    s.y = y;
    return MR_OK;
}

// Launch with programmatic stream serialization (see pdl_trigger / pdl_wait).
template <typename... Params, typename... Args>
int launch(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MR_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...));
    return MR_OK;
}

// The probe slots of the next probed launch (tracing only), else NULL.
unsigned long long *next_probe(HeavyEngine &e) {
    if (!e.probes || e.probe_n >= e.probe_cap) return nullptr;
    return e.probes + static_cast<size_t>(kProbeSlots) * e.probe_n++;
}

// A stamp after the kernel just queued (tracing only).
int stamp(HeavyEngine &e) {
    if (!e.trace || e.trace_n >= e.trace_cap) return MR_OK;
    return launch(k_stamp, 1, 32, 0, e.stream, e.trace + e.trace_n++);
}

int launch_gemv(HeavyEngine &e, std::initializer_list<GemvSeg> segs) {
    GemvArgs a{};
    int blocks = 0, cols = 0;
    for (const GemvSeg &s : segs) {
        a.first[a.nseg] = blocks;
        a.s[a.nseg++] = s;
        blocks += (s.rows + kGemvRows - 1) / kGemvRows;
        cols = std::max(cols, s.cols);
    }
    a.first[a.nseg] = blocks;
    if (int rc = launch(k_gemv, blocks, kGemvThreads, static_cast<size_t>(cols) * sizeof(float) + 16, e.stream, a))
        return rc;
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

}  // namespace

int heavy_create(mr_model *m, const mr_model_config &c, cudaStream_t stream, const float *inv_freq_host, int rank,
                 int ranks, HeavyEngine **out) {
    auto *e = new HeavyEngine();
    e->rank = rank;
    e->ranks = ranks;
    e->m = m;
    e->stream = stream;
    e->H = c.query_heads;
    e->KVH = c.kv_heads;
    e->d = c.head_dim;
    e->hidden = c.hidden_size;
    e->latent = c.latent_dim;
    e->ffn = c.ffn_dim;
    e->vocab = c.vocab_size;
    e->layers = c.layers;
    e->loops = std::max(1, c.inner_loop_steps);
    e->context = c.context_length;
    e->window = c.window;
    e->block = c.block_size;
    e->slots = c.global_slots;
    e->experts = c.routed_experts;
    e->groups = c.router_groups;
    e->per_group = (c.routed_experts + c.router_groups - 1) / c.router_groups;
    e->max_k = c.router_top_k_max;
    e->min_k = c.router_top_k_min;
    e->shared = c.shared_experts;
    e->split_half = c.split_half_rope;
    e->tied = c.tie_embeddings;
    e->eps = c.norm_eps;
    e->residual_scale = c.residual_scale;
    e->temperature = c.router_temperature;
    e->slope = c.alibi_slope;
    e->log_experts = static_cast<float>(std::log(static_cast<double>(c.routed_experts)));
    auto fail = [&](int rc) {
        heavy_destroy(e);
        return rc;
    };
    if (!(e->window > 0 && e->block > 0 && e->latent > 0 && e->experts > 0 && e->experts <= 256 && e->groups > 0 &&
          e->max_k >= 1 && e->max_k <= 64 && e->min_k >= 0 && e->slots >= 0 && e->shared >= 0 &&
          e->H % e->KVH == 0 && e->d <= 1024 && e->d % 2 == 0 && e->d / 2 <= 128)) {
        heavy_destroy(e);
        return set_error(MR_ERR_ARGUMENT, "heavy-medium-2.0 geometry outside the device path's limits");
    }
    const int width = e->KVH * e->d;
    int64_t rows = 0, cols = 0;
    int rc = MR_OK;
    if ((rc = tensor_of(m, "embed", &e->embed, &e->embed_dt, &rows, &cols))) return fail(rc);
    if ((rc = tensor_of(m, "norm", &e->final_norm, &e->final_norm_dt, &rows, &cols))) return fail(rc);
    if ((rc = tensor_of(m, e->tied ? "embed" : "output", &e->head, &e->head_dt, &rows, &cols))) return fail(rc);
    // work buffers
    const int maxblocks = (e->context + e->block - 1) / e->block;
    const int slots_total = e->max_k + e->shared;
    if ((rc = halloc_n(*e, e->hidden, &e->x)) || (rc = halloc_n(*e, std::max(e->hidden, e->ffn), &e->h)) ||
        (rc = halloc_n(*e, static_cast<size_t>(e->H) * e->d, &e->q)) || (rc = halloc_n(*e, e->latent, &e->lat)) ||
        (rc = halloc_n(*e, 2 * static_cast<size_t>(width), &e->kv)) ||
        (rc = halloc_n(*e, static_cast<size_t>(e->H) * e->d, &e->attn)) ||
        (rc = halloc_n(*e, static_cast<size_t>(e->H) * (std::min(e->window, e->context) + maxblocks), &e->scores)) ||
        (rc = halloc_n(*e, e->groups + e->experts, &e->router)) ||
        (rc = halloc_n(*e, static_cast<size_t>(slots_total) * e->ffn, &e->act)) ||
        (rc = halloc_n(*e, static_cast<size_t>(slots_total) * e->hidden, &e->eout)) ||
        (rc = halloc_n(*e, e->vocab, &e->logits)) || (rc = halloc_n(*e, e->d / 2, &e->inv_freq)) ||
        (rc = halloc_n(*e, e->context + 1, &e->log1p_table)))
        return fail(rc);
    const size_t per = static_cast<size_t>(e->layers) * e->loops;
    if ((rc = halloc_n(*e, per * e->H * std::max(1, e->slots), &e->kept)) ||
        (rc = halloc_n(*e, per * e->max_k, &e->chosen)) || (rc = halloc_n(*e, per * e->max_k, &e->weights)) ||
        (rc = halloc_n(*e, per, &e->active)) || (rc = halloc_n(*e, 1, &e->d_token)) ||
        (rc = halloc_n(*e, 1, &e->err)))
        return fail(rc);
    MR_CUDA_TRY(cudaMemset(e->err, 0, sizeof(int)));
    if (ranks > 1) {
        if (ranks > kMaxHeavyRanks) {
            heavy_destroy(e);
            return set_error(MR_ERR_ARGUMENT, "at most %d ranks", kMaxHeavyRanks);
        }
        e->out_bytes = (static_cast<size_t>(slots_total) * e->hidden * sizeof(float) + 255) & ~size_t(255);
        e->flags_offset = 2 * e->out_bytes;
        e->arena_bytes = e->flags_offset + 256;
        void *arena = nullptr;
        if ((rc = halloc(*e, e->arena_bytes, &arena))) return fail(rc);
        e->arena = static_cast<char *>(arena);
        MR_CUDA_TRY(cudaMemset(e->arena, 0, e->arena_bytes));
        e->peers[rank] = e->arena;
    }
    MR_CUDA_TRY(cudaMemcpy(e->inv_freq, inv_freq_host, sizeof(float) * (e->d / 2), cudaMemcpyHostToDevice));
    for (size_t i = 0; i < per; ++i) {
        float *kr, *vr, *km, *vm;
        if ((rc = halloc_n(*e, static_cast<size_t>(e->context) * width, &kr)) ||
            (rc = halloc_n(*e, static_cast<size_t>(e->context) * width, &vr)) ||
            (rc = halloc_n(*e, static_cast<size_t>(maxblocks) * width, &km)) ||
            (rc = halloc_n(*e, static_cast<size_t>(maxblocks) * width, &vm)))
            return fail(rc);
        e->k_ring.push_back(kr);
        e->v_ring.push_back(vr);
        e->k_mean.push_back(km);
        e->v_mean.push_back(vm);
    }
    // per-layer weights
    e->L.resize(e->layers);
    for (int l = 0; l < e->layers; ++l) {
        HeavyLayer &Ly = e->L[l];
        const std::string p = "layers." + std::to_string(l) + ".";
        if ((rc = tensor_of(m, p + "a_norm", &Ly.a_norm, &Ly.a_norm_dt, &rows, &cols)) ||
            (rc = tensor_of(m, p + "f_norm", &Ly.f_norm, &Ly.f_norm_dt, &rows, &cols)) ||
            (rc = seg_of(m, p + "q", e->h, e->q, Ly.q)) || (rc = seg_of(m, p + "latent", e->h, e->lat, Ly.latent)) ||
            (rc = seg_of(m, p + "kv_up", e->lat, e->kv, Ly.kv_up)) || (rc = seg_of(m, p + "o", e->attn, e->x, Ly.o)) ||
            (rc = seg_of(m, p + "router.coarse.weight", e->h, e->router, Ly.coarse)) ||
            (rc = seg_of(m, p + "router.fine.weight", e->h, e->router + e->groups, Ly.fine)) ||
            (rc = tensor_of(m, p + "router.coarse.bias", &Ly.coarse_bias, &Ly.bias_dt[0], &rows, &cols)) ||
            (rc = tensor_of(m, p + "router.group_bias", &Ly.group_bias, &Ly.bias_dt[1], &rows, &cols)) ||
            (rc = tensor_of(m, p + "router.fine.bias", &Ly.fine_bias, &Ly.bias_dt[2], &rows, &cols)) ||
            (rc = tensor_of(m, p + "router.expert_bias", &Ly.expert_bias, &Ly.bias_dt[3], &rows, &cols)))
            return fail(rc);
        Ly.o.residual = 1;
        for (GemvSeg *g : {&Ly.q, &Ly.latent, &Ly.coarse, &Ly.fine}) {  // inputs: RMSNorm(x, a_norm / f_norm)
            const bool attention = g == &Ly.q || g == &Ly.latent;
            g->x = e->x;
            g->norm = 1;
            g->gain = attention ? Ly.a_norm : Ly.f_norm;
            g->gain_dtype = attention ? Ly.a_norm_dt : Ly.f_norm_dt;
            g->eps = e->eps;
        }
        std::vector<const void *> gate, up, down;
        int dtype = -1;
        for (int i = 0; i < e->experts + e->shared; ++i) {
            const std::string root = i < e->experts ? p + "experts." + std::to_string(i) + "."
                                                    : p + "shared." + std::to_string(i - e->experts) + ".";
            const void *g, *u, *dn;
            int dg, du, dd;
            if ((rc = tensor_of(m, root + "gate", &g, &dg, &rows, &cols)) ||
                (rc = tensor_of(m, root + "up", &u, &du, &rows, &cols)) ||
                (rc = tensor_of(m, root + "down", &dn, &dd, &rows, &cols)))
                return fail(rc);
            if (dtype < 0) dtype = dg;
            if (dg != dtype || du != dtype || dd != dtype) {
                heavy_destroy(e);
                return set_error(MR_ERR_ARGUMENT, "layer %d: the experts' matrices must share one dtype", l);
            }
            gate.push_back(g);
            up.push_back(u);
            down.push_back(dn);
        }
        Ly.expert_dtype = dtype;
        Ly.h_gate = gate;
        Ly.h_up = up;
        Ly.h_down = down;
        const size_t n = gate.size();
        if ((rc = halloc_n(*e, n, &Ly.d_gate)) || (rc = halloc_n(*e, n, &Ly.d_up)) ||
            (rc = halloc_n(*e, n, &Ly.d_down)))
            return fail(rc);
        MR_CUDA_TRY(cudaMemcpy(Ly.d_gate, gate.data(), n * sizeof(void *), cudaMemcpyHostToDevice));
        MR_CUDA_TRY(cudaMemcpy(Ly.d_up, up.data(), n * sizeof(void *), cudaMemcpyHostToDevice));
        MR_CUDA_TRY(cudaMemcpy(Ly.d_down, down.data(), n * sizeof(void *), cudaMemcpyHostToDevice));
    }
    // fused attention and streaming kernels
    {
        int dev = 0;
        MR_CUDA_TRY(cudaGetDevice(&dev));
        MR_CUDA_TRY(cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, dev));
        MR_CUDA_TRY(cudaDeviceGetAttribute(&e->smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
        MR_CUDA_TRY(cudaDeviceGetAttribute(&e->smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
        const int G = e->H / e->KVH;
        if (G > attn::kMaxG || e->d % 4 != 0 || e->d > attn::kMaxDim) {
            heavy_destroy(e);
            return set_error(MR_ERR_ARGUMENT, "heavy-medium-2.0: %d query heads per KV head and head_dim %d are "
                             "outside the fused attention's limits (<= %d, a multiple of 4 up to %d)",
                             G, e->d, attn::kMaxG, attn::kMaxDim);
        }
        e->attn_chunks = (std::min(e->window, e->context) + attn::kChunk - 1) / attn::kChunk;
        const size_t units = static_cast<size_t>(e->attn_chunks) + 1;
        if ((rc = halloc_n(*e, e->KVH * units * G * (e->d + 2), &e->attn_partial)) ||
            (rc = halloc_n(*e, 2 * static_cast<size_t>(e->KVH) + 1, &e->counters)))
            return fail(rc);
        for (size_t i = 0; i < per; ++i) {
            float *ks, *vs;
            if ((rc = halloc_n(*e, width, &ks)) || (rc = halloc_n(*e, width, &vs))) return fail(rc);
            e->k_bsum.push_back(ks);
            e->v_bsum.push_back(vs);
        }
        const size_t attn_smem =
            attn::smem_bytes(e->latent, G, e->d, maxblocks, std::max(1, e->slots), e->attn_chunks);
        MR_REQUIRE(static_cast<size_t>(G) * std::max(1, e->slots) * e->d <= static_cast<size_t>(attn::kChunk) * e->d,
                   "heavy-medium-2.0: %d kept blocks per query head exceed the attention tiles", e->slots);
        MR_CUDA_TRY(cudaFuncSetAttribute(attn::k_sparse_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(attn_smem)));
        // the streaming kernel needs rows of whole 16-byte chunks and one dtype per launch
        auto whole = [](const GemvSeg &g) { return ((static_cast<size_t>(g.cols) * (g.dtype == MR_DTYPE_F32 ? 4 : 2)) & 15) == 0; };
        bool ok = ((static_cast<size_t>(e->hidden) * (e->head_dt == MR_DTYPE_F32 ? 4 : 2)) & 15) == 0;
        for (const HeavyLayer &Ly : e->L) {
            ok = ok && whole(Ly.q) && whole(Ly.latent) && whole(Ly.o) && Ly.q.dtype == Ly.latent.dtype;
            const size_t eb = Ly.expert_dtype == MR_DTYPE_F32 ? 4 : 2;
            ok = ok && ((e->hidden * eb) & 15) == 0 && ((e->ffn * eb) & 15) == 0;
        }
        ok = ok && slots_total <= stream::kMaxSegs;
        e->streamable = ok;
        // the batched prompt: BF16 matrices whose rows are whole 16-byte pieces, one engine
        // (the routed experts of other ranks are not here), limits of its attention kernel
        bool batch = e->ranks == 1 && e->head_dt == MR_DTYPE_BF16 && e->hidden % 8 == 0 && e->latent % 8 == 0 &&
                     e->ffn % 8 == 0 && (e->H * e->d) % 8 == 0 && e->slots <= hp::kMaxSlots && G <= hp::kRows &&
                     e->experts <= 256 && e->max_k <= 64;
        for (const HeavyLayer &Ly : e->L)
            for (const GemvSeg *g : {&Ly.q, &Ly.latent, &Ly.kv_up, &Ly.o, &Ly.coarse, &Ly.fine})
                batch = batch && g->dtype == MR_DTYPE_BF16;
        for (const HeavyLayer &Ly : e->L) batch = batch && Ly.expert_dtype == MR_DTYPE_BF16;
        batch = batch && hp::attention_smem(e->d, maxblocks) <= 227 * 1024;
        e->batchable = batch;
        for (auto kernel : {stream::k_stream<MR_DTYPE_BF16>, stream::k_stream<MR_DTYPE_F16>,
                            stream::k_stream<MR_DTYPE_F32>})
            MR_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStreamSmem));
    }
    MR_CUDA_TRY(cudaMemset(e->kept, 0xff, per * e->H * std::max(1, e->slots) * sizeof(int)));
    MR_CUDA_TRY(cudaMemset(e->chosen, 0xff, per * e->max_k * sizeof(int)));
    MR_CUDA_TRY(cudaMemset(e->weights, 0, per * e->max_k * sizeof(float)));
    MR_CUDA_TRY(cudaMemset(e->active, 0, per * sizeof(int)));
    *out = e;
    return MR_OK;
}

void heavy_destroy(HeavyEngine *e) {
    if (!e) return;
    for (void *p : e->batch.buffers) cudaFree(p);
    for (void *p : e->allocations) cudaFree(p);
    delete e;
}

int heavy_set_wait_limit(HeavyEngine *e, unsigned long long nanoseconds) {
    e->wait_ns = nanoseconds;
    return MR_OK;
}

int heavy_inject_fault(HeavyEngine *e, bool on) {
    e->withhold = on;
    return MR_OK;
}

int heavy_reset(HeavyEngine *e) {
    MR_CUDA_TRY(cudaMemset(e->counters, 0, (2 * static_cast<size_t>(e->KVH) + 1) * sizeof(unsigned long long)));
    MR_CUDA_TRY(cudaMemset(e->err, 0, sizeof(int)));
    if (e->batch.err) MR_CUDA_TRY(cudaMemset(e->batch.err, 0, sizeof(int)));
    e->attn_seq = e->route_seq = 0;
    return MR_OK;
}

int heavy_set_log1p(HeavyEngine *e, const float *values, int n) {
    MR_REQUIRE(e && values, "NULL argument");
    MR_REQUIRE(n >= e->context, "the log1p table needs %d values (distances 0 .. context-1), got %d", e->context, n);
    MR_CUDA_TRY(cudaMemcpy(e->log1p_table, values, sizeof(float) * e->context, cudaMemcpyHostToDevice));
    e->table_set = true;
    return MR_OK;
}

// One token at `position`: x = embed[token], every layer and inner loop, the
// final norm and the head; logits (vocab floats) stay in e->logits.
namespace {
int token_step(HeavyEngine *e, const int *dtoken, int token, int position);
}

int heavy_token(HeavyEngine *e, int token, int position) {
    MR_REQUIRE(token >= 0 && token < e->vocab, "input token is outside the vocabulary");
    return token_step(e, nullptr, token, position);
}

int heavy_token_from_slot(HeavyEngine *e, int position) { return token_step(e, e->d_token, 0, position); }
int *heavy_token_slot(HeavyEngine *e) { return e->d_token; }

int heavy_greedy_chain(HeavyEngine *e, int first_token, int position, int steps) {
    MR_REQUIRE(first_token >= 0 && first_token < e->vocab, "input token is outside the vocabulary");
    for (int i = 0; i < steps; ++i) {
        if (int rc = token_step(e, i ? e->d_token : nullptr, first_token, position + i)) return rc;
        if (int rc = launch(k_argmax, 1, 1024, 0, e->stream, e->logits, e->vocab, e->d_token)) return rc;
    }
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

namespace {

// Launches k_stream for one dtype; the ring takes the shared memory the
// launch's other regions leave.
// `beside`: the shared memory of the previous kernel's CTA.  When a ring of at
// least kMinBeside slots still lets a CTA of this launch sit beside one of
// those on an SM, the ring is cut to that size, so that this launch's CTAs
// start streaming while the previous kernel runs (the o projection after the
// attention: 7 slots instead of 12).
constexpr int kMinBeside = 6;
int launch_stream(HeavyEngine &e, stream::Args a, size_t beside = 0) {
    const int grid = e.sm_count;
    const size_t fixed = stream::fixed_smem(a, grid);
    a.slot_bytes = stream::slot_bytes(a);
    const int slots = static_cast<int>((kStreamSmem - fixed) / a.slot_bytes);
    MR_REQUIRE(slots >= 2, "streaming GEMV: %zu bytes of inputs leave no room for the weight ring", fixed);
    a.probe = next_probe(e);
    a.wait_ns = e.wait_ns;
    a.slots = std::min({slots, stream::kMaxSlots, e.stream_slots[a.mode]});
    if (beside) {
        const long long room = static_cast<long long>(e.smem_per_sm) - 2LL * e.smem_reserved -
                               static_cast<long long>(beside) - static_cast<long long>(fixed);
        const int fit = room > 0 ? static_cast<int>(room / a.slot_bytes) : 0;
        if (fit >= kMinBeside) a.slots = std::min(a.slots, fit);
    }
    MR_REQUIRE(a.residual == 0 || a.nseg == 1, "streaming GEMV: a residual launch has one matrix");
    a.err = e.err;
    const size_t smem = fixed + static_cast<size_t>(a.slots) * a.slot_bytes;
    switch (a.dtype) {
        case MR_DTYPE_BF16: return launch(stream::k_stream<MR_DTYPE_BF16>, grid, stream::kThreads, smem, e.stream, a);
        case MR_DTYPE_F16: return launch(stream::k_stream<MR_DTYPE_F16>, grid, stream::kThreads, smem, e.stream, a);
        default: return launch(stream::k_stream<MR_DTYPE_F32>, grid, stream::kThreads, smem, e.stream, a);
    }
}

// y = W x (or y += scale W x) for matrices of one width and dtype, the input
// RMSNorm'ed with `gain` when given.
int stream_plain(HeavyEngine &e, std::initializer_list<GemvSeg> segs, const float *x, const void *gain,
                 int gain_dtype, int residual, float scale, size_t beside = 0) {
    stream::Args a{};
    a.mode = stream::kPlain;
    for (const GemvSeg &g : segs) {
        a.dtype = g.dtype;
        a.cols = g.cols;
        a.seg[a.nseg++] = stream::Seg{g.w, nullptr, g.y, g.rows, 0};
    }
    a.x = x;
    a.norm = gain != nullptr;
    a.gain = gain;
    a.gain_dtype = gain_dtype;
    a.eps = e.eps;
    a.residual = residual;
    a.scale = scale;
    return launch_stream(e, a, beside);
}

int token_step(HeavyEngine *e, const int *dtoken, int token, int position) {
    MR_REQUIRE(e->table_set, "heavy-medium-2.0: the distance-penalty table has not been set");
    MR_REQUIRE(position >= 0 && position < e->context, "position %d outside the context", position);
    cudaStream_t s = e->stream;
    const int count = position + 1;
    const int length = std::min(e->window, count), start = count - length;
    const int blocks = (count + e->block - 1) / e->block;
    const int slots = std::min(e->slots, blocks);
    const int slots_total = e->max_k + e->shared;
    const int G = e->H / e->KVH;
    const int maxblocks = (e->context + e->block - 1) / e->block;
    const float loop_scale = static_cast<float>(static_cast<double>(e->residual_scale) / std::sqrt((double)e->loops));
    const float shared_scale = static_cast<float>(static_cast<double>(e->residual_scale) / std::max(e->shared, 1));
    const size_t attn_smem =
        attn::smem_bytes(e->latent, G, e->d, maxblocks, std::max(1, e->slots), e->attn_chunks);
    if (int rc = launch(k_embed_row, (e->hidden + 255) / 256, 256, 0, s, e->embed, e->embed_dt, dtoken, token,
                        e->hidden, e->x))
        return rc;
    if (int rc = stamp(*e)) return rc;
    for (int l = 0; l < e->layers; ++l) {
        HeavyLayer &Ly = e->L[l];
        for (int loop = 0; loop < e->loops; ++loop) {
            const size_t li = static_cast<size_t>(l) * e->loops + loop;
            // 1. q | latent of RMSNorm(x, a_norm)
            if (e->streamable) {
                if (int rc = stream_plain(*e, {Ly.q, Ly.latent}, e->x, Ly.a_norm, Ly.a_norm_dt, 0, 1.0f)) return rc;
            } else if (int rc = launch_gemv(*e, {Ly.q, Ly.latent})) {
                return rc;
            }
            if (int rc = stamp(*e)) return rc;
            // 2. sparse attention (model.py:192-229) in one launch
            attn::Args aa{};
            aa.q = e->q;
            aa.latent = e->lat;
            aa.kv_up = Ly.kv_up.w;
            aa.kv_dtype = Ly.kv_up.dtype;
            aa.latent_dim = e->latent;
            aa.kv = e->kv;
            aa.k_ring = e->k_ring[li];
            aa.v_ring = e->v_ring[li];
            aa.k_mean = e->k_mean[li];
            aa.v_mean = e->v_mean[li];
            aa.k_bsum = e->k_bsum[li];
            aa.v_bsum = e->v_bsum[li];
            aa.inv_freq = e->inv_freq;
            aa.split_half = e->split_half;
            aa.H = e->H;
            aa.KVH = e->KVH;
            aa.d = e->d;
            aa.position = position;
            aa.count = count;
            aa.length = length;
            aa.start = start;
            aa.blocks = blocks;
            aa.block = e->block;
            aa.slots = slots;
            aa.slots_max = std::max(1, e->slots);
            aa.chunks = e->attn_chunks;
            aa.max_blocks = maxblocks;
            aa.log1p_table = e->log1p_table;
            aa.slope = e->slope;
            aa.kept = e->kept + li * e->H * std::max(1, e->slots);
            aa.partial = e->attn_partial;
            aa.ready = e->counters;
            aa.wdone = e->counters + e->KVH;
            aa.seq = ++e->attn_seq;
            aa.out = e->attn;
            aa.err = e->err;
            aa.probe = next_probe(*e);
            aa.wait_ns = e->wait_ns;
            aa.withhold = e->withhold;
            if (int rc = launch(attn::k_sparse_attention, e->KVH * (e->attn_chunks + 1), attn::kThreads, attn_smem, s,
                                aa))
                return rc;
            if (int rc = stamp(*e)) return rc;
            // 3. x += s * W_o attended
            if (e->streamable) {
                if (int rc = stream_plain(*e, {Ly.o}, e->attn, nullptr, 0, 1, loop_scale, attn_smem)) return rc;
            } else {
                GemvSeg o = Ly.o;
                o.scale = loop_scale;
                if (int rc = launch_gemv(*e, {o})) return rc;
            }
            if (int rc = stamp(*e)) return rc;
            // 4. router logits of RMSNorm(x, f_norm), then the routing (model.py:231-250)
            RouteArgs ra{};
            ra.router = e->router;
            ra.coarse_bias = Ly.coarse_bias;
            ra.group_bias = Ly.group_bias;
            ra.fine_bias = Ly.fine_bias;
            ra.expert_bias = Ly.expert_bias;
            for (int i = 0; i < 4; ++i) ra.bias_dtype[i] = Ly.bias_dt[i];
            ra.experts = e->experts;
            ra.groups = e->groups;
            ra.per_group = e->per_group;
            ra.max_k = e->max_k;
            ra.min_k = e->min_k;
            ra.temperature = e->temperature;
            ra.log_experts = e->log_experts;
            ra.chosen = e->chosen + li * e->max_k;
            ra.weights = e->weights + li * e->max_k;
            ra.active = e->active + li;
            RouterArgs rt{};
            rt.ra = ra;
            rt.logits = e->router;
            rt.coarse = Ly.coarse.w;
            rt.fine = Ly.fine.w;
            rt.dtype = Ly.coarse.dtype;
            rt.cols = e->hidden;
            rt.groups = e->groups;
            rt.experts = e->experts;
            rt.x = e->x;
            rt.gain = Ly.f_norm;
            rt.gain_dtype = Ly.f_norm_dt;
            rt.eps = e->eps;
            rt.done = e->counters + 2 * e->KVH;
            rt.seq = ++e->route_seq;
            rt.probe = next_probe(*e);
            const int router_blocks = (e->groups + e->experts + kGemvRows - 1) / kGemvRows;
            if (int rc = launch(k_router_route, router_blocks, kGemvThreads,
                                static_cast<size_t>(e->hidden) * sizeof(float) + 16, s, rt))
                return rc;
            if (int rc = stamp(*e)) return rc;
            // 5-6. the chosen and the shared experts, then the rank-order combine (model.py:251-255);
            // expert parallel: this rank's experts, their rows to every rank, then the combine
            unsigned long long tag = 0;
            size_t out_offset = 0;
            if (e->ranks > 1) {  // this step's half of the arena (the other half: the step before)
                tag = ++e->moe_tag;
                out_offset = (tag & 1) * e->out_bytes;
            }
            auto mine = [&](int expert) { return e->ranks == 1 || expert % e->ranks == e->rank; };
            if (e->streamable) {
                stream::Args g{};
                g.mode = stream::kSwiglu;
                g.dtype = Ly.expert_dtype;
                g.cols = e->hidden;
                for (int i = 0; i < e->shared; ++i)
                    if (mine(e->experts + i))
                        g.seg[g.nseg++] = stream::Seg{Ly.h_gate[e->experts + i], Ly.h_up[e->experts + i], nullptr,
                                                      e->ffn, e->max_k + i};
                g.rank = e->rank;
                g.ranks = e->ranks;
                g.dyn_w = Ly.d_gate;
                g.dyn_w2 = Ly.d_up;
                g.chosen = ra.chosen;
                g.active = ra.active;
                g.max_k = e->max_k;
                g.dyn_rows = e->ffn;
                g.experts = e->experts;
                g.shared = e->shared;
                g.x = e->x;
                g.norm = 1;
                g.gain = Ly.f_norm;
                g.gain_dtype = Ly.f_norm_dt;
                g.eps = e->eps;
                g.act_out = e->act;
                if (int rc = launch_stream(*e, g)) return rc;
                if (int rc = stamp(*e)) return rc;
                stream::Args dn{};
                dn.mode = stream::kDown;
                dn.dtype = Ly.expert_dtype;
                dn.cols = e->ffn;
                for (int i = 0; i < e->shared; ++i)
                    if (mine(e->experts + i))
                        dn.seg[dn.nseg++] = stream::Seg{Ly.h_down[e->experts + i], nullptr, nullptr, e->hidden,
                                                        e->max_k + i};
                dn.rank = e->rank;
                dn.ranks = e->ranks;
                dn.out_offset = out_offset;
                for (int j = 0; j < e->ranks && e->ranks > 1; ++j) dn.peer[j] = e->peers[j];
                dn.dyn_w = Ly.d_down;
                dn.chosen = ra.chosen;
                dn.active = ra.active;
                dn.max_k = e->max_k;
                dn.dyn_rows = e->hidden;
                dn.experts = e->experts;
                dn.shared = e->shared;
                dn.acts = e->act;
                dn.weights = ra.weights;
                dn.shared_scale = shared_scale;
                dn.scale = loop_scale;
                dn.xres = e->x;
                if (int rc = launch_stream(*e, dn)) return rc;
                if (int rc = stamp(*e)) return rc;
                if (e->ranks == 1) continue;
            }
            ExpertArgs ea{};
            ea.gate = Ly.d_gate;
            ea.up = Ly.d_up;
            ea.down = Ly.d_down;
            ea.dtype = Ly.expert_dtype;
            ea.ffn = e->ffn;
            ea.hidden = e->hidden;
            ea.experts = e->experts;
            ea.max_k = e->max_k;
            ea.shared = e->shared;
            ea.chosen = ra.chosen;
            ea.active = ra.active;
            ea.x = e->x;
            ea.norm_gain = Ly.f_norm;
            ea.norm_dtype = Ly.f_norm_dt;
            ea.eps = e->eps;
            ea.act = e->act;
            ea.out = e->eout;
            ea.rank = e->rank;
            ea.ranks = e->ranks;
            ea.err = e->err;
            ea.wait_ns = e->wait_ns;
            if (e->ranks > 1) {
                ea.tag = tag;
                ea.out_offset = out_offset;
                ea.out = reinterpret_cast<float *>(e->arena + ea.out_offset);
                ea.flags = reinterpret_cast<unsigned long long *>(e->arena + e->flags_offset);
                ea.flags_offset = e->flags_offset;
                for (int j = 0; j < e->ranks; ++j) ea.peer[j] = e->peers[j];
            }
            if (!e->streamable) {  // rows that are not whole 16-byte pieces: the per-expert kernels
                if (int rc = launch(k_expert_gate_up, dim3((e->ffn + 7) / 8, slots_total), kGemvThreads,
                                    static_cast<size_t>(e->hidden) * sizeof(float) + 16, s, ea))
                    return rc;
                if (int rc = stamp(*e)) return rc;
                if (int rc = launch(k_expert_down, dim3((e->hidden + kGemvRows - 1) / kGemvRows, slots_total),
                                    kGemvThreads, static_cast<size_t>(e->ffn) * sizeof(float) + 16, s, ea))
                    return rc;
                if (int rc = stamp(*e)) return rc;
            }
            if (e->ranks > 1) {
                if (int rc = launch(k_moe_publish, 1, 32, 0, s, ea)) return rc;
                if (int rc = stamp(*e)) return rc;
            }
            if (int rc = launch(k_expert_combine, (e->hidden + 255) / 256, 256, 0, s, ea, ra.weights, shared_scale,
                                loop_scale, e->x))
                return rc;
            if (int rc = stamp(*e)) return rc;
        }
    }
    // the head of RMSNorm(x, norm)
    GemvSeg head{};
    head.w = e->head;
    head.dtype = e->head_dt;
    head.rows = e->vocab;
    head.cols = e->hidden;
    head.x = e->x;
    head.y = e->logits;
    head.norm = 1;
    head.gain = e->final_norm;
    head.gain_dtype = e->final_norm_dt;
    head.eps = e->eps;
    if (e->streamable) {
        if (int rc = stream_plain(*e, {head}, e->x, e->final_norm, e->final_norm_dt, 0, 1.0f)) return rc;
    } else if (int rc = launch_gemv(*e, {head})) {
        return rc;
    }
    if (int rc = stamp(*e)) return rc;
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}
}  // namespace

const float *heavy_logits(const HeavyEngine *e) { return e->logits; }

int heavy_trace_token(HeavyEngine *e, int token, int position, unsigned long long *stamps, int capacity, int *count) {
    MR_REQUIRE(token >= 0 && token < e->vocab, "input token is outside the vocabulary");
    MR_REQUIRE(stamps && count && capacity >= 2, "NULL argument or no room for stamps");
    // layout of `stamps`: [0 .. kernels] kernel-boundary stamps, then kProbeSlots per probed launch
    const int probed = 6 * e->layers * e->loops + 1;
    const int nstamps = std::max(2, capacity - probed * kProbeSlots);
    unsigned long long *d = nullptr;
    MR_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void **>(&d), sizeof(unsigned long long) * capacity, e->stream));
    MR_CUDA_TRY(cudaMemsetAsync(d, 0, sizeof(unsigned long long) * capacity, e->stream));
    const bool with_probes = capacity >= nstamps + probed * kProbeSlots;
    if (with_probes) {  // minima start at the largest value
        std::vector<unsigned long long> init(static_cast<size_t>(probed) * kProbeSlots, 0ull);
        for (int i = 0; i < probed; ++i) init[static_cast<size_t>(i) * kProbeSlots + kProbeStart] =
            init[static_cast<size_t>(i) * kProbeSlots + kProbeWaited] = ~0ull;
        MR_CUDA_TRY(cudaMemcpyAsync(d + nstamps, init.data(), init.size() * sizeof(unsigned long long),
                                    cudaMemcpyHostToDevice, e->stream));
        MR_CUDA_TRY(cudaStreamSynchronize(e->stream));
        e->probes = d + nstamps;
        e->probe_n = 0;
        e->probe_cap = probed;
    }
    e->trace = d;
    e->trace_n = 0;
    e->trace_cap = nstamps;
    int rc = stamp(*e);  // the step's start: the work queued before it has completed
    if (!rc) rc = token_step(e, nullptr, token, position);
    const int n = e->trace_n;
    e->trace = e->probes = nullptr;
    e->trace_n = e->trace_cap = e->probe_n = e->probe_cap = 0;
    cudaError_t err = cudaStreamSynchronize(e->stream);
    if (!rc && err == cudaSuccess)
        err = cudaMemcpy(stamps, d, sizeof(unsigned long long) * capacity, cudaMemcpyDeviceToHost);
    cudaFreeAsync(d, e->stream);
    if (rc) return rc;
    if (err != cudaSuccess) return cuda_error(err, "heavy trace");
    *count = n;
    return MR_OK;
}

void heavy_arena(const HeavyEngine *e, char **arena, size_t *bytes) {
    *arena = e->arena;
    *bytes = e->arena_bytes;
}

void heavy_connect(HeavyEngine *e, char *const *peers) {
    for (int j = 0; j < e->ranks; ++j) e->peers[j] = peers[j];
}


// ---- batched prompt (heavy_prefill.cuh) ---------------------------------------------------
namespace {

void batch_release(HeavyBatch &b) {
    for (void *p : b.buffers) cudaFree(p);
    b = HeavyBatch{};
}

// Grows the workspace to chunks of `tokens` tokens; on first use also the
// per-layer router matrices and expert weight maps.
int batch_reserve(HeavyEngine &e, int tokens, bool all_logits) {
    HeavyBatch &b = e.batch;
    if (b.ready && b.cap >= tokens && (b.all_logits || !all_logits)) return MR_OK;
    const int T = std::max(tokens, b.cap);
    const bool all = all_logits || b.all_logits;
    batch_release(b);
    const int h = e.hidden, qd = e.H * e.d, width = e.KVH * e.d, f = e.ffn, E = e.experts, K = e.max_k;
    const size_t R = static_cast<size_t>(T) * K;
    b.kmax = std::max({h, qd, e.latent, f});
    b.max_tiles = static_cast<int>(R / kBatchTileRows) + E + 1;
    auto get = [&](size_t bytes, auto **out) -> int {
        void *p = nullptr;
        MR_CUDA_TRY(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
        b.buffers.push_back(p);
        *out = static_cast<std::remove_reference_t<decltype(**out)> *>(p);
        return MR_OK;
    };
    const size_t f4 = sizeof(float), u2 = sizeof(uint16_t), i4 = sizeof(int);
    int rc = get(T * i4, &b.ids);
    if (!rc) rc = get(i4, &b.err);
    if (!rc) rc = get(f4 * T * h, &b.x);
    if (!rc) rc = get(u2 * 3 * static_cast<size_t>(T) * b.kmax, &b.planes);
    if (!rc) rc = get(f4 * T * static_cast<size_t>(qd + e.latent), &b.qlat);
    if (!rc) rc = get(f4 * T * 2 * static_cast<size_t>(width), &b.kv);
    if (!rc) rc = get(f4 * T * static_cast<size_t>(qd), &b.qh);
    if (!rc) rc = get(f4 * T * static_cast<size_t>(width), &b.sum_k);
    if (!rc) rc = get(f4 * T * static_cast<size_t>(width), &b.sum_v);
    if (!rc) rc = get(f4 * T * static_cast<size_t>(e.groups + E), &b.rlog);
    if (!rc) rc = get(i4 * R, &b.chosen);
    if (!rc) rc = get(f4 * R, &b.weights);
    if (!rc) rc = get(i4 * T, &b.active);
    if (!rc) rc = get(i4 * R, &b.row_of);
    if (!rc) rc = get(i4 * R, &b.token_of);
    if (!rc) rc = get(4 * i4 * static_cast<size_t>(b.max_tiles), &b.tiles);
    if (!rc) rc = get(i4, &b.tile_count);
    if (!rc) rc = get(i4, &b.rows);
    if (!rc) rc = get(u2 * 3 * R * h, &b.gplanes);
    if (!rc) rc = get(f4 * R * 2 * f, &b.gu);
    if (!rc) rc = get(u2 * 3 * R * f, &b.gsplanes);
    if (!rc) rc = get(f4 * R * h, &b.rout);
    if (!rc) rc = get(f4 * T * 2 * static_cast<size_t>(f) * std::max(1, e.shared), &b.sgu);
    if (!rc) rc = get(f4 * T * static_cast<size_t>(h) * std::max(1, e.shared), &b.sout);
    if (!rc) rc = get(f4 * (all ? T : 1) * static_cast<size_t>(e.vocab), &b.logits);
    b.window_tc = e.d == hp::kWDim && hp::kWRows % (e.H / e.KVH) == 0;
    if (!rc && b.window_tc) rc = get(f4 * T * static_cast<size_t>(e.H) * (e.d + 2), &b.bstate);
    if (!rc && b.window_tc)
        rc = get(hp::kTileBytes * e.KVH * static_cast<size_t>((T + e.window) / hp::kWKeys + 2), &b.kv_planes);
    // per layer: coarse | fine router rows as one matrix, the experts' weight maps
    const size_t router_rows = static_cast<size_t>(e.groups) + E;
    if (!rc) rc = get(u2 * router_rows * h * e.layers, &b.router_w);
    if (!rc) rc = get(kBatchMapBytes * 2 * E * static_cast<size_t>(e.layers), &b.maps_gu);
    if (!rc) rc = get(kBatchMapBytes * E * static_cast<size_t>(e.layers), &b.maps_dn);
    if (rc) {
        batch_release(b);
        return rc;
    }
    std::vector<unsigned char> gu(kBatchMapBytes * 2 * E * e.layers), dn(kBatchMapBytes * E * e.layers);
    for (int l = 0; l < e.layers && !rc; ++l) {
        const HeavyLayer &Ly = e.L[l];
        uint16_t *rw = b.router_w + static_cast<size_t>(l) * router_rows * h;
        const cudaError_t c1 = cudaMemcpyAsync(rw, Ly.coarse.w, u2 * e.groups * h, cudaMemcpyDeviceToDevice, e.stream);
        const cudaError_t c2 =
            cudaMemcpyAsync(rw + static_cast<size_t>(e.groups) * h, Ly.fine.w, u2 * E * h, cudaMemcpyDeviceToDevice, e.stream);
        if (c1 != cudaSuccess || c2 != cudaSuccess) rc = set_error(MR_ERR_CUDA, "router rows copy failed");
        for (int x = 0; x < E && !rc; ++x) {
            const size_t at = static_cast<size_t>(l) * E + x;
            rc = batch_weight_map(gu.data() + (2 * at) * kBatchMapBytes, Ly.h_gate[x], f, h);
            if (!rc) rc = batch_weight_map(gu.data() + (2 * at + 1) * kBatchMapBytes, Ly.h_up[x], f, h);
            if (!rc) rc = batch_weight_map(dn.data() + at * kBatchMapBytes, Ly.h_down[x], h, f);
        }
    }
    if (!rc && (cudaMemcpy(b.maps_gu, gu.data(), gu.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(b.maps_dn, dn.data(), dn.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemset(b.err, 0, sizeof(int)) != cudaSuccess))
        rc = set_error(MR_ERR_CUDA, "batched prompt setup failed");
    if (!rc) rc = batch_setup();
    if (!rc)
        MR_CUDA_TRY(cudaFuncSetAttribute(hp::k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(hp::attention_smem(e.d, (e.context + e.block - 1) / e.block))));
    if (!rc && b.window_tc)
        MR_CUDA_TRY(cudaFuncSetAttribute(hp::k_window_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(hp::kWindowSmem)));
    if (rc) {
        batch_release(b);
        return rc;
    }
    b.cap = T;
    b.all_logits = all;
    b.ready = true;
    return MR_OK;
}

int grid_for(size_t n, int threads = 256) {
    return static_cast<int>(std::min<size_t>((n + threads - 1) / threads, 148 * 16));
}

}  // namespace

bool heavy_batchable(const HeavyEngine *e) { return e->batchable; }
const float *heavy_prefill_logits(const HeavyEngine *e) { return e->batch.logits; }

int heavy_prefill(HeavyEngine *e, const int *ids, int T, int p0, bool all_logits) {
    MR_REQUIRE(e->batchable, "heavy-medium-2.0: this model does not qualify for the batched prompt");
    MR_REQUIRE(e->table_set, "heavy-medium-2.0: the distance-penalty table has not been set");
    MR_REQUIRE(T > 0 && p0 >= 0 && p0 + T <= e->context, "positions %d .. %d outside the context", p0, p0 + T - 1);
    for (int i = 0; i < T; ++i) MR_REQUIRE(ids[i] >= 0 && ids[i] < e->vocab, "input token is outside the vocabulary");
    if (int rc = batch_reserve(*e, T, all_logits)) return rc;
    HeavyBatch &b = e->batch;
    cudaStream_t s = e->stream;
    const int h = e->hidden, H = e->H, d = e->d, qd = H * d, lat = e->latent, KVH = e->KVH, width = KVH * d;
    const int f = e->ffn, E = e->experts, K = e->max_k, G = H / KVH, RG = e->groups + E;
    const size_t ps = static_cast<size_t>(b.cap) * b.kmax;           // plane strides
    const size_t R = static_cast<size_t>(b.cap) * K;
    const size_t gps = R * h, gsps = R * f;
    const int ldq = qd + lat, slots_max = std::max(1, e->slots);
    const float loop_scale = static_cast<float>(static_cast<double>(e->residual_scale) / std::sqrt((double)e->loops));
    const float shared_scale = static_cast<float>(static_cast<double>(e->residual_scale) / std::max(e->shared, 1));
    const int nb = (p0 + T - 1) / e->block + 1;
    MR_CUDA_TRY(cudaMemcpyAsync(b.ids, ids, sizeof(int) * T, cudaMemcpyHostToDevice, s));
    hp::k_embed<<<T, 256, 0, s>>>(b.ids, T, e->embed, e->embed_dt, h, b.x);
    MR_CUDA_TRY(cudaGetLastError());
    int rc = MR_OK;
    for (int l = 0; l < e->layers && !rc; ++l) {
        const HeavyLayer &Ly = e->L[l];
        for (int loop = 0; loop < e->loops && !rc; ++loop) {
            const size_t li = static_cast<size_t>(l) * e->loops + loop;
            // q | latent of RMSNorm(x, a_norm); kv = W_kv_up latent
            rc = batch_rms_planes(s, b.x, 0, T, h, h, Ly.a_norm, Ly.a_norm_dt, e->eps, b.planes, ps, b.kmax);
            const BatchSeg ql[2] = {{Ly.q.w, qd, 0}, {Ly.latent.w, lat, qd}};
            if (!rc) rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, T, h, ql, 2, b.qlat, ldq, false, 0.f);
            if (rc) break;
            hp::k_split<<<grid_for(static_cast<size_t>(T) * lat), 256, 0, s>>>(b.qlat + qd, ldq, lat, T, b.planes, ps,
                                                                               b.kmax);
            const BatchSeg kvs = {Ly.kv_up.w, 2 * width, 0};
            rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, T, lat, &kvs, 1, b.kv, 2 * width, false, 0.f);
            if (rc) break;
            // queries, keys and values at the chunk's positions; block sums and means
            hp::k_qk<<<(T * (H + 2 * KVH) * 32 + 255) / 256, 256, 0, s>>>(b.qlat, ldq, b.kv, T, p0, H, KVH, d,
                                                                           e->split_half, e->inv_freq, b.qh, e->k_ring[li],
                                                                           e->v_ring[li]);
            hp::k_block_sums<<<grid_for(static_cast<size_t>((p0 + T - 1) / e->block - p0 / e->block + 1) * width * 2),
                               256, 0, s>>>(e->k_ring[li], e->v_ring[li], T, p0, width, e->block, e->k_bsum[li],
                                            e->v_bsum[li], e->k_mean[li], e->v_mean[li], b.sum_k, b.sum_v);
            // sparse attention of every token -> planes of the o projection's input
            hp::AttnArgs aa{};
            aa.qh = b.qh;
            aa.k_rows = e->k_ring[li];
            aa.v_rows = e->v_ring[li];
            aa.k_mean = e->k_mean[li];
            aa.v_mean = e->v_mean[li];
            aa.sum_k = b.sum_k;
            aa.sum_v = b.sum_v;
            aa.log1p_table = e->log1p_table;
            aa.slope = e->slope;
            aa.T = T;
            aa.p0 = p0;
            aa.H = H;
            aa.KVH = KVH;
            aa.d = d;
            aa.window = e->window;
            aa.block = e->block;
            aa.slots = e->slots;
            aa.slots_max = slots_max;
            aa.nb = nb;
            aa.planes = b.planes;
            aa.ps = ps;
            aa.ld = b.kmax;
            aa.kept_last = e->kept + li * H * slots_max;
            aa.block_state = b.window_tc ? b.bstate : nullptr;  // the window part then runs on tcgen05
            const int QT = hp::kRows / G;
            hp::k_attention<<<dim3((T + QT - 1) / QT, KVH), hp::kThreads, hp::attention_smem(d, nb), s>>>(aa);
            MR_CUDA_TRY(cudaGetLastError());
            if (b.window_tc) {
                // the 64-key blocks from the first one a window of the chunk reaches to the chunk's end
                const int block0 = std::max(0, p0 - e->window + 1) / hp::kWKeys;
                const int nblocks = (p0 + T - 1) / hp::kWKeys - block0 + 1;
                hp::k_kv_planes<<<nblocks * KVH, 256, 0, s>>>(e->k_ring[li], e->v_ring[li], KVH, block0, p0 + T,
                                                              b.kv_planes);
                MR_CUDA_TRY(cudaGetLastError());
                hp::WindowArgs wa{};
                wa.qh = b.qh;
                wa.kv_planes = b.kv_planes;
                wa.block0 = block0;
                wa.block_state = b.bstate;
                wa.T = T;
                wa.p0 = p0;
                wa.H = H;
                wa.KVH = KVH;
                wa.d = d;
                wa.window = e->window;
                wa.planes = b.planes;
                wa.ps = ps;
                wa.ld = b.kmax;
                wa.err = b.err;
                const int WT = hp::kWRows / G;
                hp::k_window_tc<<<dim3((T + WT - 1) / WT, KVH), hp::kWThreads, hp::kWindowSmem, s>>>(wa);
                MR_CUDA_TRY(cudaGetLastError());
            }
            // x += s W_o attended
            const BatchSeg os = {Ly.o.w, h, 0};
            rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, T, qd, &os, 1, b.x, h, true, loop_scale);
            // router logits of RMSNorm(x, f_norm) and the routing of every token
            if (!rc) rc = batch_rms_planes(s, b.x, 0, T, h, h, Ly.f_norm, Ly.f_norm_dt, e->eps, b.planes, ps, b.kmax);
            const BatchSeg rs = {b.router_w + static_cast<size_t>(l) * RG * h, RG, 0};
            if (!rc) rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, T, h, &rs, 1, b.rlog, RG, false, 0.f);
            if (rc) break;
            hp::RouteRows rr{};
            rr.ra.router = b.rlog;
            rr.ra.coarse_bias = Ly.coarse_bias;
            rr.ra.group_bias = Ly.group_bias;
            rr.ra.fine_bias = Ly.fine_bias;
            rr.ra.expert_bias = Ly.expert_bias;
            for (int i = 0; i < 4; ++i) rr.ra.bias_dtype[i] = Ly.bias_dt[i];
            rr.ra.experts = E;
            rr.ra.groups = e->groups;
            rr.ra.per_group = e->per_group;
            rr.ra.max_k = K;
            rr.ra.min_k = e->min_k;
            rr.ra.temperature = e->temperature;
            rr.ra.log_experts = e->log_experts;
            rr.ra.chosen = b.chosen;
            rr.ra.weights = b.weights;
            rr.ra.active = b.active;
            rr.ld_router = RG;
            rr.T = T;
            hp::k_route<<<T, 256, 0, s>>>(rr);
            // the routed rows sorted by expert, gathered; grouped gate | up, SwiGLU, down
            hp::k_moe_plan<<<1, 1024, 0, s>>>(b.chosen, b.active, T, K, E, b.row_of, b.token_of,
                                              reinterpret_cast<int4 *>(b.tiles), b.tile_count, b.max_tiles, b.rows,
                                              e->err);
            hp::k_gather<<<grid_for(R * (h / 8) * 3 / 4), 256, 0, s>>>(b.planes, ps, b.kmax, b.token_of, b.rows, h,
                                                                       b.gplanes, gps, h);
            MR_CUDA_TRY(cudaGetLastError());
            const BatchSeg gus[2] = {{nullptr, f, 0}, {nullptr, f, f}};
            rc = batch_gemm_grouped(s, b.err, b.gplanes, gps, h, static_cast<int>(R), h,
                                    b.maps_gu + static_cast<size_t>(l) * E * 2 * kBatchMapBytes, gus, 2, b.tiles,
                                    b.tile_count, b.max_tiles, b.gu, 2 * f);
            if (rc) break;
            hp::k_swiglu<<<grid_for(R * f / 4), 256, 0, s>>>(b.gu, b.rows, 0, f, b.gsplanes, gsps, f);
            const BatchSeg dns = {nullptr, h, 0};
            rc = batch_gemm_grouped(s, b.err, b.gsplanes, gsps, f, static_cast<int>(R), f,
                                    b.maps_dn + static_cast<size_t>(l) * E * kBatchMapBytes, &dns, 1, b.tiles,
                                    b.tile_count, b.max_tiles, b.rout, h);
            // the shared experts over every token (their gate | up first: the planes are reused)
            for (int j = 0; j < e->shared && !rc; ++j) {
                const BatchSeg sg[2] = {{Ly.h_gate[E + j], f, 0}, {Ly.h_up[E + j], f, f}};
                rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, T, h, sg, 2,
                                b.sgu + static_cast<size_t>(j) * T * 2 * f, 2 * f, false, 0.f);
            }
            for (int j = 0; j < e->shared && !rc; ++j) {
                hp::k_swiglu<<<grid_for(static_cast<size_t>(T) * f), 256, 0, s>>>(
                    b.sgu + static_cast<size_t>(j) * T * 2 * f, nullptr, T, f, b.planes, ps, b.kmax);
                const BatchSeg sd = {Ly.h_down[E + j], h, 0};
                rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, T, f, &sd, 1, b.sout + static_cast<size_t>(j) * T * h, h,
                                false, 0.f);
            }
            if (rc) break;
            hp::k_combine<<<grid_for(static_cast<size_t>(T) * h), 256, 0, s>>>(
                b.x, T, h, b.active, b.weights, b.row_of, K, b.rout, b.sout, e->shared, shared_scale, loop_scale);
            MR_CUDA_TRY(cudaGetLastError());
            // the last token's experts, where the token step leaves its own
            MR_CUDA_TRY(cudaMemcpyAsync(e->chosen + li * K, b.chosen + static_cast<size_t>(T - 1) * K, sizeof(int) * K,
                                        cudaMemcpyDeviceToDevice, s));
            MR_CUDA_TRY(cudaMemcpyAsync(e->weights + li * K, b.weights + static_cast<size_t>(T - 1) * K,
                                        sizeof(float) * K, cudaMemcpyDeviceToDevice, s));
            MR_CUDA_TRY(cudaMemcpyAsync(e->active + li, b.active + T - 1, sizeof(int), cudaMemcpyDeviceToDevice, s));
        }
    }
    if (rc) return rc;
    // final RMSNorm and the head for the rows whose logits are wanted
    const int r0 = all_logits ? 0 : T - 1, rows = all_logits ? T : 1;
    rc = batch_rms_planes(s, b.x, r0, rows, h, h, e->final_norm, e->final_norm_dt, e->eps, b.planes, ps, b.kmax);
    const BatchSeg hs = {e->head, e->vocab, 0};
    if (!rc) rc = batch_gemm(s, b.err, b.planes, ps, b.kmax, rows, h, &hs, 1, b.logits, e->vocab, false, 0.f);
    return rc;
}

int heavy_status(const HeavyEngine *e) {
    int err = 0;
    MR_CUDA_TRY(cudaMemcpy(&err, e->err, sizeof(int), cudaMemcpyDeviceToHost));
    switch (err) {
        case 0: break;
        case 1: return set_error(MR_ERR_TIMEOUT, "expert parallel: a rank's expert rows did not arrive within the wait limit");
        case 2: return set_error(MR_ERR_TIMEOUT, "weight stream: a bulk copy did not land within the wait limit");
        case 3: return set_error(MR_ERR_TIMEOUT, "sparse attention: a key / value row did not arrive within the wait limit");
        case 4: return set_error(MR_ERR_CUDA, "expert routing chose an id outside the expert table (non-finite router "
                                              "logits?)");
        default: return set_error(MR_ERR_TIMEOUT, "heavy-medium-2.0: device wait timed out (code %d)", err);
    }
    if (e->batch.err) {
        MR_CUDA_TRY(cudaMemcpy(&err, e->batch.err, sizeof(int), cudaMemcpyDeviceToHost));
        if (err) return set_error(MR_ERR_TIMEOUT, "batched prompt: a GEMM's bounded wait gave up");
    }
    return MR_OK;
}

int heavy_last_topk(const HeavyEngine *e, int layer, int loop, int *blocks, int capacity) {
    const int per = e->H * std::max(1, e->slots);
    MR_REQUIRE(capacity >= e->H * e->slots, "blocks holds %d ints, need %d", capacity, e->H * e->slots);
    std::vector<int> tmp(per);
    MR_CUDA_TRY(cudaStreamSynchronize(e->stream));
    MR_CUDA_TRY(cudaMemcpy(tmp.data(), e->kept + (static_cast<size_t>(layer) * e->loops + loop) * per,
                           sizeof(int) * per, cudaMemcpyDeviceToHost));
    for (int i = 0; i < e->H * e->slots; ++i) blocks[i] = tmp[i];
    return MR_OK;
}

int heavy_last_experts(const HeavyEngine *e, int layer, int loop, int *experts, float *weights, int capacity) {
    MR_REQUIRE(capacity >= e->max_k, "buffers hold %d entries, need %d", capacity, e->max_k);
    const size_t li = static_cast<size_t>(layer) * e->loops + loop;
    MR_CUDA_TRY(cudaStreamSynchronize(e->stream));
    MR_CUDA_TRY(cudaMemcpy(experts, e->chosen + li * e->max_k, sizeof(int) * e->max_k, cudaMemcpyDeviceToHost));
    MR_CUDA_TRY(cudaMemcpy(weights, e->weights + li * e->max_k, sizeof(float) * e->max_k, cudaMemcpyDeviceToHost));
    return MR_OK;
}

}  // namespace mr
