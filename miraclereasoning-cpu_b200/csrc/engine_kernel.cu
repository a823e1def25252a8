// Persistent decode kernel: one cooperative launch per token, one CTA per SM,
// every phase of the step separated by a bounded grid barrier.
//
// Reference semantics per phase:
//   GEMV      model._linear / kernels.cl linear (5-17), RMSNorm of the input
//             (kernels.cl rms, 19-28), residual axpy (52-56), SwiGLU (46-50)
//   ATTN_GQA  model._gqa (model.py:95-116): per-head Q/K RMSNorm, RoPE
//             (kernels.cl:30-44), ring append (model.py:21-25), scores /
//             softmax / mix over the ring in logical order plus relay rows
//             (kernels.cl:58-107)
//
// Numerics: weights are widened from their stored dtype exactly as the
// reference widens them; all arithmetic is float32.  Dot products and the
// softmax use tree/online reductions, so logits match the reference within
// float32 rounding (the parity tests pin atol 2e-5 / rtol 2e-4), not bit for
// bit.  Element-wise steps (residual, SwiGLU, RoPE) round each product and sum
// separately, as FP_CONTRACT OFF does in the reference.
#include "engine.cuh"

namespace mr {
namespace {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr int kKeyTile = 32;
constexpr size_t kPrefetchCap = 512 * 1024;  // bytes of next-phase weights per CTA

struct Shared {
    float in[kMaxInput];
    float partial[kEngineWarps * kEngineWarps];
    float y[kMaxSegments][kRowBatch];
    float red[kEngineWarps];
    float merge_w[kMergeSlots];
    unsigned long long best[kEngineWarps];
    int flag;
    int ok;
};

struct StepInfo {
    int position, token, logits_row;
};

__device__ __forceinline__ void row_range(int rows, int b, int g, int &r0, int &r1) {
    r0 = static_cast<int>(static_cast<long long>(rows) * b / g);
    r1 = static_cast<int>(static_cast<long long>(rows) * (b + 1) / g);
}

__device__ __forceinline__ int esize(int dtype) { return dtype == MR_DTYPE_F32 ? 4 : 2; }

// ---- grid barrier ------------------------------------------------------------------
// Arrive, then wait (thread 0 of each CTA) until every CTA has arrived.  The
// wait is bounded: after kWaitLimitNs it records 1000+phase in st->error and
// every CTA returns, leaving the context usable.
__device__ bool grid_barrier(StepState *st, unsigned long long target, int phase, Shared &sm) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        atomicAdd(&st->barrier, 1ull);
        uint64_t start = 0;
        for (unsigned spin = 0;; ++spin) {
            if (ld_acquire_u64(&st->barrier) >= target) break;
            if ((spin & 63u) == 63u) {
                if (*reinterpret_cast<volatile int *>(&st->error)) {
                    ok = 0;
                    break;
                }
                const uint64_t now = global_ns();
                if (!start) {
                    start = now;
                } else if (now - start > kWaitLimitNs) {
                    atomicCAS(&st->error, 0, 1000 + phase);
                    ok = 0;
                    break;
                }
            }
        }
        __threadfence();
        sm.ok = ok;
    }
    __syncthreads();
    return sm.ok != 0;
}

// Deterministic block sum (same order in every CTA -> identical bits).
__device__ float block_sum(float v, Shared &sm) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sm.red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float total = lane < kEngineWarps ? sm.red[lane] : 0.f;
        total = warp_sum(total);
        if (lane == 0) sm.red[0] = total;
    }
    __syncthreads();
    const float total = sm.red[0];
    __syncthreads();
    return total;
}

// ---- GEMV --------------------------------------------------------------------------
// One 16-byte chunk of a weight row times the matching shared-memory inputs.
template <int DT>
struct RowDot;

template <>
struct RowDot<MR_DTYPE_BF16> {
    static constexpr int VEC = 8;
    __device__ static float chunk(const uint4 &w, const float *x) {
        const float4 a = *reinterpret_cast<const float4 *>(x), b = *reinterpret_cast<const float4 *>(x + 4);
        float acc = __uint_as_float(w.x << 16) * a.x;
        acc = fmaf(__uint_as_float(w.x & 0xffff0000u), a.y, acc);
        acc = fmaf(__uint_as_float(w.y << 16), a.z, acc);
        acc = fmaf(__uint_as_float(w.y & 0xffff0000u), a.w, acc);
        acc = fmaf(__uint_as_float(w.z << 16), b.x, acc);
        acc = fmaf(__uint_as_float(w.z & 0xffff0000u), b.y, acc);
        acc = fmaf(__uint_as_float(w.w << 16), b.z, acc);
        acc = fmaf(__uint_as_float(w.w & 0xffff0000u), b.w, acc);
        return acc;
    }
};

template <>
struct RowDot<MR_DTYPE_F16> {
    static constexpr int VEC = 8;
    __device__ static float chunk(const uint4 &w, const float *x) {
        const float4 a = *reinterpret_cast<const float4 *>(x), b = *reinterpret_cast<const float4 *>(x + 4);
        const __half2 *h = reinterpret_cast<const __half2 *>(&w);
        const float2 p0 = __half22float2(h[0]), p1 = __half22float2(h[1]), p2 = __half22float2(h[2]),
                     p3 = __half22float2(h[3]);
        float acc = p0.x * a.x;
        acc = fmaf(p0.y, a.y, acc);
        acc = fmaf(p1.x, a.z, acc);
        acc = fmaf(p1.y, a.w, acc);
        acc = fmaf(p2.x, b.x, acc);
        acc = fmaf(p2.y, b.y, acc);
        acc = fmaf(p3.x, b.z, acc);
        acc = fmaf(p3.y, b.w, acc);
        return acc;
    }
};

template <>
struct RowDot<MR_DTYPE_F32> {
    static constexpr int VEC = 4;
    __device__ static float chunk(const uint4 &w, const float *x) {
        const float4 a = *reinterpret_cast<const float4 *>(x);
        float acc = __uint_as_float(w.x) * a.x;
        acc = fmaf(__uint_as_float(w.y), a.y, acc);
        acc = fmaf(__uint_as_float(w.z), a.z, acc);
        acc = fmaf(__uint_as_float(w.w), a.w, acc);
        return acc;
    }
};

// Weights are read once per step: bypass L1 (they were prefetched into L2).
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Partial dot product of weight `row` with the input: 16-byte chunks
// first, first+stride, ...; elements past the last whole chunk are taken by
// lane `tail_lane` (-1: none).  Rows whose byte length is not a multiple of 16
// (tiny shapes only) fall back to scalar loads by the tail lane's warp.
template <int DT>
__device__ float row_partial(const void *wbase, int cols, int row, int first, int stride, int tail_lane,
                             const float *x) {
    using D = RowDot<DT>;
    const int nv = cols / D::VEC;
    const size_t row_bytes = static_cast<size_t>(cols) * esize(DT);
    const char *rp = static_cast<const char *>(wbase) + static_cast<size_t>(row) * row_bytes;
    float acc = 0.f;
    if ((row_bytes & 15) == 0) {
        const uint4 *v = reinterpret_cast<const uint4 *>(rp);
        int c = first;
        for (; c + 3 * stride < nv; c += 4 * stride) {
            const uint4 w0 = ld_stream(v + c), w1 = ld_stream(v + c + stride), w2 = ld_stream(v + c + 2 * stride),
                        w3 = ld_stream(v + c + 3 * stride);
            acc += D::chunk(w0, x + c * D::VEC);
            acc += D::chunk(w1, x + (c + stride) * D::VEC);
            acc += D::chunk(w2, x + (c + 2 * stride) * D::VEC);
            acc += D::chunk(w3, x + (c + 3 * stride) * D::VEC);
        }
        for (; c < nv; c += stride) acc += D::chunk(ld_stream(v + c), x + c * D::VEC);
        if (tail_lane >= 0) {
            for (int j = nv * D::VEC + tail_lane; j < cols; j += 32) acc = fmaf(load_weight(rp, DT, j), x[j], acc);
        }
    } else if (tail_lane >= 0) {
        for (int j = tail_lane; j < cols; j += 32) acc = fmaf(load_weight(rp, DT, j), x[j], acc);
    }
    return acc;
}

__device__ float row_partial_any(const Segment &s, int row, int first, int stride, int tail_lane, const float *x) {
    switch (s.dtype) {
        case MR_DTYPE_BF16: return row_partial<MR_DTYPE_BF16>(s.w, s.cols, row, first, stride, tail_lane, x);
        case MR_DTYPE_F16: return row_partial<MR_DTYPE_F16>(s.w, s.cols, row, first, stride, tail_lane, x);
        default: return row_partial<MR_DTYPE_F32>(s.w, s.cols, row, first, stride, tail_lane, x);
    }
}

// y[i] = W[r0+i] . in for i < n (n <= kRowBatch), results in sm.y[slot].
// Many rows: one warp per row.  Few rows: several warps split each row.
__device__ void gemv_rows(const Segment &s, int r0, int n, int slot, Shared &sm) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (n >= kEngineWarps) {
        for (int i = warp; i < n; i += kEngineWarps) {
            float acc = row_partial_any(s, r0 + i, lane, 32, lane, sm.in);
            acc = warp_sum(acc);
            if (lane == 0) sm.y[slot][i] = acc;
        }
        __syncthreads();
        return;
    }
    const int wpr = kEngineWarps / n;  // warps per row
    const int i = warp / wpr, part = warp % wpr;
    if (i < n) {
        float acc = row_partial_any(s, r0 + i, part * 32 + lane, 32 * wpr, part == 0 ? lane : -1, sm.in);
        acc = warp_sum(acc);
        if (lane == 0) sm.partial[i * wpr + part] = acc;
    }
    __syncthreads();
    if (threadIdx.x < n) {
        float total = 0.f;
        for (int p = 0; p < wpr; ++p) total += sm.partial[threadIdx.x * wpr + p];
        sm.y[slot][threadIdx.x] = total;
    }
    __syncthreads();
}

__device__ void load_input(const GemvPhase &g, int cols, int token, Shared &sm) {
    if (g.input_kind == IN_EMBED_ROW) {
        for (int j = threadIdx.x; j < cols; j += blockDim.x) {
            const float v = load_weight(g.embed, g.embed_dtype, static_cast<size_t>(token) * cols + j);
            sm.in[j] = v;
            if (g.embed_copy && blockIdx.x == 0) g.embed_copy[j] = v;
        }
    } else {
        for (int j = threadIdx.x; j < cols; j += blockDim.x) sm.in[j] = __ldcg(g.in + j);
    }
    __syncthreads();
    if (g.norm) {
        float ss = 0.f;
        for (int j = threadIdx.x; j < cols; j += blockDim.x) ss = fmaf(sm.in[j], sm.in[j], ss);
        ss = block_sum(ss, sm);
        // kernels.cl:25-27: scale = 1/sqrt(mean + eps); y = (x * scale) * gain
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), g.norm_eps)));
        for (int j = threadIdx.x; j < cols; j += blockDim.x) {
            const float gain = g.norm_gain ? load_weight(g.norm_gain, g.norm_gain_dtype, j) : 1.0f;
            sm.in[j] = __fmul_rn(__fmul_rn(sm.in[j], scale), gain);
        }
        __syncthreads();
    }
}

__device__ void gemv_phase(const GemvPhase &g, StepState *st, const StepInfo &info, Shared &sm) {
    const int G = gridDim.x, b = blockIdx.x;
    const int cols = g.seg[0].cols;
    load_input(g, cols, info.token, sm);
    const bool paired = g.epilogue == EPI_SWIGLU;
    const int passes = paired ? 1 : g.nseg;
    unsigned long long best = 0;
    int nonfinite = 0;
    for (int s = 0; s < passes; ++s) {
        const Segment &seg = g.seg[s];
        int r0, r1;
        row_range(seg.rows, b, G, r0, r1);
        for (int rb = r0; rb < r1; rb += kRowBatch) {
            const int n = min(kRowBatch, r1 - rb);
            gemv_rows(seg, rb, n, 0, sm);
            if (paired) gemv_rows(g.seg[1], rb, n, 1, sm);
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int r = rb + i;
                const float y = sm.y[0][i];
                switch (g.epilogue) {
                    case EPI_STORE: seg.out[r] = y; break;
                    case EPI_RESIDUAL: g.x[r] = __fadd_rn(__ldcg(g.x + r), __fmul_rn(g.scale, y)); break;
                    case EPI_SWIGLU: {
                        const float u = sm.y[1][i];
                        g.out[r] = __fmul_rn(__fdiv_rn(y, __fadd_rn(1.0f, expf(-y))), u);
                        break;
                    }
                    case EPI_LOGITS: {
                        g.out[static_cast<size_t>(info.logits_row) * seg.rows + r] = y;
                        if (!isfinite(y)) nonfinite = 1;
                        else best = max(best, argmax_key(y, r));
                        break;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (g.epilogue == EPI_LOGITS) {
        // CTA argmax -> one atomic per CTA
        for (int offset = 16; offset > 0; offset >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, offset));
        nonfinite = __any_sync(0xffffffffu, nonfinite);
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        if (lane == 0) {
            sm.best[warp] = best;
            if (nonfinite) atomicExch(&st->nonfinite, 1);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long m = 0;
            for (int w = 0; w < kEngineWarps; ++w) m = max(m, sm.best[w]);
            if (m) atomicMax(&st->best, m);
        }
        __syncthreads();
    }
}

__device__ void prefetch_gemv(const GemvPhase &g) {
    if (threadIdx.x != 0) return;
    const int G = gridDim.x, b = blockIdx.x;
    size_t budget = kPrefetchCap;
    const int nseg = g.epilogue == EPI_SWIGLU ? 2 : g.nseg;
    for (int s = 0; s < nseg && budget; ++s) {
        const Segment &seg = g.seg[s];
        int r0, r1;
        row_range(seg.rows, b, G, r0, r1);
        if (r1 <= r0) continue;
        const size_t row_bytes = static_cast<size_t>(seg.cols) * esize(seg.dtype);
        size_t bytes = static_cast<size_t>(r1 - r0) * row_bytes;
        if (bytes > budget) bytes = budget;
        budget -= bytes;
        prefetch_l2(static_cast<const char *>(seg.w) + static_cast<size_t>(r0) * row_bytes, bytes);
    }
}

// ---- grouped-query attention ------------------------------------------------------
__device__ __forceinline__ void rope_pair(float &u, float &v, float angle) {
    const float c = cosf(angle), s = sinf(angle);
    const float a = __fsub_rn(__fmul_rn(u, c), __fmul_rn(v, s));
    const float b = __fadd_rn(__fmul_rn(u, s), __fmul_rn(v, c));
    u = a;
    v = b;
}

// In-place per-head RMSNorm (optional) + RoPE of a [dim] vector held by one warp
// in shared memory (kernels.cl rms 19-28 then rope 30-44).
__device__ void norm_rope_warp(float *v, int dim, const void *gain, int gain_dtype, float eps, bool do_norm,
                               const float *inv_freq, float position, int split_half) {
    const int lane = threadIdx.x & 31;
    if (do_norm) {
        float ss = 0.f;
        for (int j = lane; j < dim; j += 32) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
        for (int j = lane; j < dim; j += 32) {
            const float gn = gain ? load_weight(gain, gain_dtype, j) : 1.0f;
            v[j] = __fmul_rn(__fmul_rn(v[j], scale), gn);
        }
        __syncwarp();
    }
    const int half = dim / 2;
    for (int p = lane; p < half; p += 32) {
        const int j = split_half ? p : 2 * p, k = split_half ? p + half : 2 * p + 1;
        float u = v[j], w = v[k];
        rope_pair(u, w, __fmul_rn(position, inv_freq[p]));
        v[j] = u;
        v[k] = w;
    }
    __syncwarp();
}

// Work unit = (KV head g, chunk c of the attended rows).  Each unit does an
// online-softmax pass over its rows for the group's query heads; a chunked
// head's partials are merged by the unit that arrives last.
__device__ void attn_gqa_phase(const AttnPhase &a, const StepInfo &info, Shared &sm) {
    const int G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = a.dim, gq = a.heads / a.kv_heads;
    const int count = info.position + 1;
    const int cap = a.capacity;
    const int length = min(count, cap);
    const int start = (count - length) % cap;
    const int extra = a.relay_count ? __ldcg(a.relay_count) : 0;
    const int total = length + extra;
    int chunks = max(1, min(a.max_chunks, G / a.kv_heads));
    chunks = min(chunks, max(1, (total + kKeyTile - 1) / kKeyTile));
    chunks = min(chunks, kMergeSlots / gq);
    const int chunk_len = (total + chunks - 1) / chunks;
    chunks = (total + chunk_len - 1) / chunk_len;
    const float pos_f = static_cast<float>(info.position);
    const float sqrt_d = __fsqrt_rn(static_cast<float>(d));  // divisor, kernels.cl:72

    // shared-memory carve-up (reuses the GEMV input area)
    float *q = sm.in;                                  // [gq][d]
    float *kt = q + gq * d;                            // [kKeyTile][d+1]
    float *vt = kt + kKeyTile * (d + 1);               // [kKeyTile][d]
    float *p = vt + kKeyTile * d;                      // [gq][kKeyTile]
    float *acc = p + gq * kKeyTile;                    // [gq][d]
    float *mrow = acc + gq * d;                        // [gq]
    float *lrow = mrow + gq;                           // [gq]
    float *corr = lrow + gq;                           // [gq]
    float *knew = corr + gq;                           // [d]

    for (int unit = blockIdx.x; unit < a.kv_heads * chunks; unit += G) {
        const int g = unit / chunks, c = unit % chunks;
        const int t0 = c * chunk_len, t1 = min(total, t0 + chunk_len);
        // 1. this group's query heads: RMSNorm + RoPE
        for (int i = warp; i < gq; i += kEngineWarps) {
            float *qi = q + i * d;
            const float *src = a.q_raw + static_cast<size_t>(g * gq + i) * d;
            for (int j = lane; j < d; j += 32) qi[j] = __ldcg(src + j);
            __syncwarp();
            norm_rope_warp(qi, d, a.q_gain, a.gain_dtype, a.norm_eps, a.qk_norm != 0, a.inv_freq, pos_f,
                           a.split_half);
        }
        // 2. the unit owning the newest ring row appends this token's key/value
        const int newest = length - 1;
        if (newest >= t0 && newest < t1) {
            const size_t slot = static_cast<size_t>(g) * cap + (count - 1) % cap;
            if (warp == 0) {
                const float *src = a.k_raw + static_cast<size_t>(g) * d;
                for (int j = lane; j < d; j += 32) knew[j] = __ldcg(src + j);
                __syncwarp();
                norm_rope_warp(knew, d, a.k_gain, a.gain_dtype, a.norm_eps, a.qk_norm != 0, a.inv_freq, pos_f,
                               a.split_half);
                for (int j = lane; j < d; j += 32) a.k_cache[slot * d + j] = knew[j];
            } else if (warp == 1) {
                const float *src = a.v_raw + static_cast<size_t>(g) * d;
                for (int j = lane; j < d; j += 32) a.v_cache[slot * d + j] = __ldcg(src + j);
            }
        }
        for (int e = threadIdx.x; e < gq * d; e += blockDim.x) acc[e] = 0.f;
        if (threadIdx.x < gq) {
            mrow[threadIdx.x] = -INFINITY;
            lrow[threadIdx.x] = 0.f;
        }
        __syncthreads();
        // 3. key tiles: scores, online softmax, value mix
        for (int tb = t0; tb < t1; tb += kKeyTile) {
            const int nt = min(kKeyTile, t1 - tb);
            for (int e = threadIdx.x; e < nt * d; e += blockDim.x) {
                const int t = e / d, j = e % d, lt = tb + t;
                const float *kr, *vr;
                if (lt < length) {
                    const size_t row = static_cast<size_t>(g) * cap + (start + lt) % cap;
                    kr = a.k_cache + row * d;
                    vr = a.v_cache + row * d;
                } else {
                    const size_t row = static_cast<size_t>(g) * a.relay_capacity + (lt - length);
                    kr = a.relay_k + row * d;
                    vr = a.relay_v + row * d;
                }
                kt[t * (d + 1) + j] = __ldcg(kr + j);
                vt[t * d + j] = __ldcg(vr + j);
            }
            __syncthreads();
            for (int i = warp; i < gq; i += kEngineWarps) {
                float s = -INFINITY;
                if (lane < nt) {
                    const float *qi = q + i * d, *kr = kt + lane * (d + 1);
                    float dot = 0.f;
                    for (int j = 0; j < d; ++j) dot = fmaf(qi[j], kr[j], dot);
                    s = __fdiv_rn(dot, sqrt_d);
                }
                const float tile_max = warp_max(s);
                const float m_old = mrow[i];
                const float m_new = fmaxf(m_old, tile_max);
                const float e = (m_new == -INFINITY) ? 0.f : expf(s - m_new);
                const float tile_sum = warp_sum(e);
                p[i * kKeyTile + lane] = e;
                if (lane == 0) {
                    const float cf = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                    corr[i] = cf;
                    lrow[i] = lrow[i] * cf + tile_sum;
                    mrow[i] = m_new;
                }
            }
            __syncthreads();
            for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
                const int i = e / d, j = e % d;
                float v = acc[e] * corr[i];
                const float *pi = p + i * kKeyTile;
                for (int t = 0; t < nt; ++t) v = fmaf(pi[t], vt[t * d + j], v);
                acc[e] = v;
            }
            __syncthreads();
        }
        // 4. publish (single chunk: final; else partial + last-arriver merge)
        if (chunks == 1) {
            for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
                const int i = e / d, j = e % d;
                a.out[static_cast<size_t>(g * gq + i) * d + j] = acc[e] / lrow[i];
            }
            __syncthreads();
            continue;
        }
        const int stride = d + 2;
        for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
            const int i = e / d, j = e % d;
            a.partial[(static_cast<size_t>(g * gq + i) * a.max_chunks + c) * stride + j] = acc[e];
        }
        if (threadIdx.x < gq) {
            float *rec = a.partial + (static_cast<size_t>(g * gq + threadIdx.x) * a.max_chunks + c) * stride;
            rec[d] = mrow[threadIdx.x];
            rec[d + 1] = lrow[threadIdx.x];
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned old = atomicAdd(a.arrivals + g, 1u);
            sm.flag = (old == static_cast<unsigned>(chunks - 1));
            if (sm.flag) {
                a.arrivals[g] = 0u;
                __threadfence();
            }
        }
        __syncthreads();
        if (sm.flag) {
            // one warp per query head: all chunk maxima / sums loaded in parallel,
            // softmax-merge weights staged in shared memory
            for (int i = warp; i < gq; i += kEngineWarps) {
                const float *base = a.partial + static_cast<size_t>(g * gq + i) * a.max_chunks * stride;
                float m = -INFINITY;
                for (int cc = lane; cc < chunks; cc += 32) m = fmaxf(m, __ldcg(base + cc * stride + d));
                m = warp_max(m);
                float den = 0.f;
                for (int cc = lane; cc < chunks; cc += 32) {
                    const float mc = __ldcg(base + cc * stride + d);
                    const float w = (mc == -INFINITY) ? 0.f : expf(mc - m);
                    sm.merge_w[i * chunks + cc] = w;
                    den = fmaf(w, __ldcg(base + cc * stride + d + 1), den);
                }
                den = warp_sum(den);
                __syncwarp();
                for (int cc = lane; cc < chunks; cc += 32) sm.merge_w[i * chunks + cc] /= den;
            }
            __syncthreads();
            for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
                const int i = e / d, j = e % d;
                const float *base = a.partial + static_cast<size_t>(g * gq + i) * a.max_chunks * stride + j;
                const float *w = sm.merge_w + i * chunks;
                float num0 = 0.f, num1 = 0.f, num2 = 0.f, num3 = 0.f;
                int cc = 0;
                for (; cc + 3 < chunks; cc += 4) {
                    num0 = fmaf(w[cc], __ldcg(base + cc * stride), num0);
                    num1 = fmaf(w[cc + 1], __ldcg(base + (cc + 1) * stride), num1);
                    num2 = fmaf(w[cc + 2], __ldcg(base + (cc + 2) * stride), num2);
                    num3 = fmaf(w[cc + 3], __ldcg(base + (cc + 3) * stride), num3);
                }
                for (; cc < chunks; ++cc) num0 = fmaf(w[cc], __ldcg(base + cc * stride), num0);
                a.out[static_cast<size_t>(g * gq + i) * d + j] = (num0 + num1) + (num2 + num3);
            }
        }
        __syncthreads();
    }
}

}  // namespace

__global__ void __launch_bounds__(kEngineThreads, 1)
    decode_step_kernel(const Phase *__restrict__ phases, int nphases, StepState *st, StepControl ctl) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Shared &sm = *reinterpret_cast<Shared *>(smem_raw);
    __shared__ StepInfo info;
    __shared__ unsigned long long base;
    __shared__ int skip, need_head;
    if (threadIdx.x == 0) {
        volatile StepState *vs = st;
        skip = vs->stopped || vs->error;
        const int pos = vs->position;
        const int rel = pos - ctl.feed_base;
        info.position = pos;
        info.token = (rel >= 0 && rel < ctl.feed_len) ? ctl.feed[rel] : vs->token;
        need_head = ctl.return_all || rel >= ctl.feed_len - 1;
        info.logits_row = ctl.return_all ? rel % ctl.logits_rows : 0;
        base = vs->barrier_base;
        if (!skip && pos >= ctl.context_length) {
            if (blockIdx.x == 0) atomicCAS(&st->error, 0, 3);
            skip = 1;
        }
        if (!skip && (info.token < 0 || info.token >= ctl.vocab_size)) {
            if (blockIdx.x == 0) atomicCAS(&st->error, 0, 4);
            skip = 1;
        }
    }
    __syncthreads();
    if (skip) return;
    if (ctl.trace && blockIdx.x == 0 && threadIdx.x == 0) ctl.trace[0] = global_ns();
    int barriers = 0;
    // warm the first weight-streaming phase
    for (int p = 0; p < nphases; ++p)
        if (phases[p].kind == PH_GEMV) {
            prefetch_gemv(phases[p].gemv);
            break;
        }
    for (int p = 0; p < nphases; ++p) {
        const Phase &ph = phases[p];
        if (ph.kind == PH_STEP_END) break;
        if (ph.layer < 0 && !need_head) continue;
        // prefetch this CTA's share of the next weight-streaming phase
        for (int q = p + 1; q < nphases; ++q) {
            if (phases[q].kind == PH_GEMV) {
                if (!(phases[q].layer < 0 && !need_head)) prefetch_gemv(phases[q].gemv);
                break;
            }
        }
        if (ph.kind == PH_GEMV) gemv_phase(ph.gemv, st, info, sm);
        else if (ph.kind == PH_ATTN_GQA) attn_gqa_phase(ph.attn, info, sm);
        unsigned long long *stamp = ctl.trace ? ctl.trace + 1 + static_cast<size_t>(barriers) * (gridDim.x + 1) : nullptr;
        if (stamp) {
            __syncthreads();
            if (threadIdx.x == 0) stamp[blockIdx.x] = global_ns();
        }
        ++barriers;
        if (!grid_barrier(st, base + static_cast<unsigned long long>(barriers) * gridDim.x, p, sm)) return;
        if (stamp && blockIdx.x == 0 && threadIdx.x == 0) stamp[gridDim.x] = global_ns();
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        volatile StepState *s = st;
        const int pos = info.position;
        const int rel = pos - ctl.feed_base;
        if (need_head) {
            const unsigned long long key = s->best;
            const int arg = key ? argmax_index(key) : -1;
            s->last_argmax = arg;
            s->best = 0ull;
            if (ctl.gen_max > 0 && rel >= ctl.feed_len - 1) {
                if (s->nonfinite) {
                    s->stopped = 1;
                } else {
                    const int n = s->gen_count;
                    if (ctl.gen_out) ctl.gen_out[n] = arg;
                    s->gen_count = n + 1;
                    s->token = arg;
                    if (arg == ctl.eos || n + 1 >= ctl.gen_max) s->stopped = 1;
                }
            }
        }
        s->position = pos + 1;
        s->barrier_base = base + static_cast<unsigned long long>(barriers) * gridDim.x;
        __threadfence();
    }
}

size_t decode_step_smem_bytes() { return sizeof(Shared); }

}  // namespace mr
