// Batched prompt processing (see prefill.cuh).
//
// Per layer, for a chunk of T tokens (model.py:257-285 for each token):
//   RMSNorm rows -> BF16x3 planes -> GEMM q|k|v -> per-head q/k RMSNorm + RoPE
//   -> causal attention over ring + chunk keys (-> planes) -> GEMM o, x += s*o
//   -> RMSNorm rows -> planes -> GEMM gate|up -> SwiGLU (-> planes)
//   -> GEMM down, x += s*down -> append the chunk's keys / values to the ring.
// Then the final RMSNorm and the lm_head GEMM for the rows whose logits are
// wanted.  Element-wise steps keep the reference's rounding (kernels.cl:19-56:
// separate multiplies and adds); reductions (sums of squares, dot products,
// softmax sums) are in FP32 in a different order than the reference's serial
// loops, within the parity tolerance.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "prefill.cuh"
#include "tcgen05.cuh"

namespace mr {
namespace {

constexpr int kBM = 64;       // GEMM tile: tokens
constexpr int kBN = 64;       // GEMM tile: output features
constexpr int kBK = 32;       // GEMM tile: reduction (two k16 steps)
constexpr int kPadK = kBK + 8;  // shared row stride (bf16): 80 bytes, conflict-free ldmatrix
constexpr int kStages = 3;
constexpr int kGemmThreads = 256;  // 8 warps: 2 (tokens) x 4 (features), warp tile 32 x 16

__device__ __forceinline__ float block_reduce_sum(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

// ---- row kernels -----------------------------------------------------------------------
// x[t] = embedding row of ids[t] (widened exactly).
__global__ void k_embed_rows(const int *ids, int T, const void *embed, int dt, int h, float *x) {
    const int t = blockIdx.x;
    if (t >= T) return;
    const size_t row = static_cast<size_t>(ids[t]) * h;
    for (int j = threadIdx.x; j < h; j += blockDim.x) x[static_cast<size_t>(t) * h + j] = load_weight(embed, dt, row + j);
}

// planes[row r - r0] = split((x[r] * scale) * gain) (kernels.cl:19-28), for rows r0 .. r0 + n - 1.
__global__ void k_rms_planes(const float *x, int r0, int h, int ldx, const void *gain, int gain_dt, float eps,
                             uint16_t *planes, size_t plane_stride, int ld) {
    __shared__ float red[32];
    const int r = r0 + blockIdx.x;
    const float *xr = x + static_cast<size_t>(r) * ldx;
    float ss = 0.f;
    for (int j = threadIdx.x; j < h; j += blockDim.x) ss = fmaf(xr[j], xr[j], ss);
    ss = block_reduce_sum(ss, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)h), eps)));
    for (int j = threadIdx.x; j < h; j += blockDim.x) {
        const float gv = gain ? load_weight(gain, gain_dt, j) : 1.0f;
        put_planes(planes, plane_stride, static_cast<size_t>(blockIdx.x) * ld + j, __fmul_rn(__fmul_rn(xr[j], scale), gv));
    }
}

// planes[t] = split(silu(gate) * up) (kernels.cl:46-50); gu[t] = gate row | up row.
__global__ void k_swiglu_planes(const float *gu, int T, int f, uint16_t *planes, size_t plane_stride, int ld) {
    const size_t n = static_cast<size_t>(T) * f;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = i / f, j = i - t * f;
        const float gv = gu[t * 2 * f + j], uv = gu[t * 2 * f + f + j];
        put_planes(planes, plane_stride, t * ld + j, __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv));
    }
}

// Per (token, head row) of q|k|v: q / k rows RMSNorm'd (q/k norm) then rotated
// (kernels.cl:30-44: angle = position * frequency); v rows copied.  One warp per
// row: rows 0..H-1 queries, H..H+KV-1 keys, H+KV..H+2KV-1 values.
__global__ void k_qk_rope(const float *qkv, int T, int p0, int H, int KV, int d, int ldqkv, int qk_norm,
                          const void *q_gain, const void *k_gain, int gain_dt, float eps, const float *inv_freq,
                          int split_half, float *qh, float *kc, float *vc) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int rows = H + 2 * KV;
    if (warp >= T * rows) return;
    const int t = warp / rows, r = warp - t * rows;
    const float *src;
    float *dst;
    const void *gain = nullptr;
    bool rotate = true;
    if (r < H) {
        src = qkv + static_cast<size_t>(t) * ldqkv + static_cast<size_t>(r) * d;
        dst = qh + (static_cast<size_t>(t) * H + r) * d;
        gain = q_gain;
    } else if (r < H + KV) {
        src = qkv + static_cast<size_t>(t) * ldqkv + static_cast<size_t>(H + (r - H)) * d;
        dst = kc + (static_cast<size_t>(t) * KV + (r - H)) * d;
        gain = k_gain;
    } else {
        src = qkv + static_cast<size_t>(t) * ldqkv + static_cast<size_t>(H + KV + (r - H - KV)) * d;
        dst = vc + (static_cast<size_t>(t) * KV + (r - H - KV)) * d;
        rotate = false;
    }
    if (!rotate) {
        for (int j = lane; j < d; j += 32) dst[j] = src[j];
        return;
    }
    float scale = 1.0f;
    if (qk_norm) {
        float ss = 0.f;
        for (int j = lane; j < d; j += 32) ss = fmaf(src[j], src[j], ss);
        ss = warp_sum(ss);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
    }
    auto val = [&](int j) {
        if (!qk_norm) return src[j];
        return __fmul_rn(__fmul_rn(src[j], scale), gain ? load_weight(gain, gain_dt, j) : 1.0f);
    };
    const int half = d / 2;
    const float pos = static_cast<float>(p0 + t);
    for (int p = lane; p < half; p += 32) {
        const int j = split_half ? p : 2 * p, k = split_half ? p + half : 2 * p + 1;
        const float angle = __fmul_rn(pos, inv_freq[p]);
        const float c = cosf(angle), s = sinf(angle);
        const float u = val(j), v = val(k);
        dst[j] = __fsub_rn(__fmul_rn(u, c), __fmul_rn(v, s));
        dst[k] = __fadd_rn(__fmul_rn(u, s), __fmul_rn(v, c));
    }
}

// ---- causal attention over the ring and the chunk ------------------------------------------
constexpr int kAttnThreads = 256;
constexpr int kAttnRows = 32;  // query rows per CTA (tokens x group heads)
constexpr int kKT = 32;        // keys per tile (one per lane in the softmax step)

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}

// CTA = (block of QT tokens, KV head g), rows r = (token, group head).  Token t
// at position p = p0 + t attends to positions (p - capacity, p]: those below p0
// from the ring (slot = position % capacity), the rest from the chunk (model.py
// :95-116; the ring holds min(count, capacity) keys).  Online softmax over key
// tiles, double-buffered (the next tile loads with cp.async while the current
// one is used).  Register blocking keeps shared-memory traffic below the
// arithmetic: a thread scores 1 row x 4 keys (strided by 8) from float4 loads and
// accumulates 2-row x 4-dim output blocks (two for head dims above 64) in
// registers across the tiles; each warp updates the softmax state of its four
// rows together.  The output rows go out as BF16x3 planes of the o
// projection's input.  Head dims are multiples of 4.
__global__ void __launch_bounds__(kAttnThreads) k_attention(const float *qh, const float *kc, const float *vc,
                                                            const float *k_cache, const float *v_cache, int T, int p0,
                                                            int H, int KV, int d, int cap, int QT, uint16_t *planes,
                                                            size_t plane_stride, int ld) {
    extern __shared__ __align__(16) float sm[];
    const int gq = H / KV, g = blockIdx.y, t0 = blockIdx.x * QT;
    const int nt = min(QT, T - t0), R = nt * gq;
    const int ks = d + 4;
    float *q = sm;                         // [kAttnRows][d + 4]
    float *kt = q + kAttnRows * ks;        // [2][kKT][d + 4]
    float *vt = kt + 2 * kKT * ks;         // [2][kKT][d]
    float *s = vt + 2 * kKT * d;           // [kAttnRows][kKT + 1]
    float *mrow = s + kAttnRows * (kKT + 1);
    float *lrow = mrow + kAttnRows;
    float *corr = lrow + kAttnRows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int dq = d / 4;
    const int p_first = p0 + t0, p_last = p0 + t0 + nt - 1;
    const int lo = max(0, p_first - cap + 1);
    auto issue = [&](int kb, int buf) {  // keys kb .. kb + 31 into buffer buf (rows past the last key: not loaded)
        const int nk = min(kKT, p_last + 1 - kb);
        for (int e = tid; e < nk * dq; e += kAttnThreads) {
            const int kk = e / dq, j = (e - kk * dq) * 4, pos = kb + kk;
            const float *ksrc, *vsrc;
            if (pos < p0) {
                const size_t row = (static_cast<size_t>(g) * cap + pos % cap) * d + j;
                ksrc = k_cache + row;
                vsrc = v_cache + row;
            } else {
                const size_t row = (static_cast<size_t>(pos - p0) * KV + g) * d + j;
                ksrc = kc + row;
                vsrc = vc + row;
            }
            cp_async16(kt + (buf * kKT + kk) * ks + j, ksrc);
            cp_async16(vt + (buf * kKT + kk) * d + j, vsrc);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(lo, 0);
    for (int e = tid; e < kAttnRows * d; e += kAttnThreads) {
        const int r = e / d, j = e - r * d, tt = r / gq, i = r - tt * gq;
        q[r * ks + j] = r < R ? qh[(static_cast<size_t>(t0 + tt) * H + g * gq + i) * d + j] : 0.f;
    }
    for (int r = tid; r < kAttnRows; r += kAttnThreads) {
        mrow[r] = -INFINITY;
        lrow[r] = 0.f;
    }
    // score block: row sr, keys sk, sk + 8, sk + 16, sk + 24 (the eight key threads of a
    // row read eight consecutive key rows: distinct banks with the d + 4 row stride)
    const int sr = tid >> 3, sk = tid & 7;
    const int nblk = (kAttnRows / 2) * dq;               // output blocks: 2 rows x 4 dims
    float acc[2][8];
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[b][e] = 0.f;
    const float sqrt_d = __fsqrt_rn(static_cast<float>(d));
    int buf = 0;
    for (int kb = lo; kb <= p_last; kb += kKT, buf ^= 1) {
        const int nk = min(kKT, p_last + 1 - kb);
        if (kb + kKT <= p_last) {
            issue(kb + kKT, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // tile buf (and, first time, q and the softmax state) visible
        const float *ktb = kt + buf * kKT * ks, *vtb = vt + buf * kKT * d;
        {  // scores: 1 row x 4 keys per thread
            float a[4] = {0.f, 0.f, 0.f, 0.f};
            for (int j = 0; j < d; j += 4) {
                const float4 q0 = *reinterpret_cast<const float4 *>(q + sr * ks + j);
#pragma unroll
                for (int y = 0; y < 4; ++y) {
                    const float4 kv = *reinterpret_cast<const float4 *>(ktb + (sk + 8 * y) * ks + j);
                    a[y] = fmaf(q0.x, kv.x, fmaf(q0.y, kv.y, fmaf(q0.z, kv.z, fmaf(q0.w, kv.w, a[y]))));
                }
            }
            const int p = p_first + sr / gq;
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int kk = sk + 8 * y, pos = kb + kk;
                const bool live = sr < R && kk < nk && pos <= p && pos > p - cap;
                s[sr * (kKT + 1) + kk] = live ? __fdiv_rn(a[y], sqrt_d) : -INFINITY;  // kernels.cl:72
            }
        }
        __syncthreads();
        {  // online softmax: warp w updates rows w, w + 8, w + 16, w + 24 together, one key per lane
            float v[4], mt[4], pr[4], sum[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                v[x] = s[(warp + 8 * x) * (kKT + 1) + lane];
                mt[x] = v[x];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int x = 0; x < 4; ++x) mt[x] = fmaxf(mt[x], __shfl_xor_sync(0xffffffffu, mt[x], o));
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                const int r = warp + 8 * x;
                const float m_new = fmaxf(mrow[r], mt[x]);
                pr[x] = (v[x] == -INFINITY) ? 0.f : expf(v[x] - m_new);
                sum[x] = pr[x];
                mt[x] = m_new;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int x = 0; x < 4; ++x) sum[x] += __shfl_xor_sync(0xffffffffu, sum[x], o);
            __syncwarp();
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                const int r = warp + 8 * x;
                s[r * (kKT + 1) + lane] = pr[x];
                if (lane == 0) {
                    const float m_old = mrow[r];
                    const float cf = (m_old == -INFINITY) ? 0.f : expf(m_old - mt[x]);
                    corr[r] = cf;
                    lrow[r] = fmaf(lrow[r], cf, sum[x]);
                    mrow[r] = mt[x];
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < 2; ++b) {  // value mix: 2 rows x 4 dims per block
            const int blk = tid + b * kAttnThreads;
            if (blk >= nblk) continue;
            const int r0 = (blk / dq) * 2, j0 = (blk % dq) * 4;
            if (r0 >= R) continue;
            const float c0 = corr[r0], c1 = corr[r0 + 1];
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                acc[b][y] *= c0;
                acc[b][4 + y] *= c1;
            }
            const float *s0 = s + r0 * (kKT + 1), *s1 = s0 + (kKT + 1);
            for (int kk = 0; kk < nk; ++kk) {
                const float4 vv = *reinterpret_cast<const float4 *>(vtb + kk * d + j0);
                const float p0v = s0[kk], p1v = s1[kk];
                acc[b][0] = fmaf(p0v, vv.x, acc[b][0]);
                acc[b][1] = fmaf(p0v, vv.y, acc[b][1]);
                acc[b][2] = fmaf(p0v, vv.z, acc[b][2]);
                acc[b][3] = fmaf(p0v, vv.w, acc[b][3]);
                acc[b][4] = fmaf(p1v, vv.x, acc[b][4]);
                acc[b][5] = fmaf(p1v, vv.y, acc[b][5]);
                acc[b][6] = fmaf(p1v, vv.z, acc[b][6]);
                acc[b][7] = fmaf(p1v, vv.w, acc[b][7]);
            }
        }
        __syncthreads();  // every reader of buffer buf is done before it is refilled
    }
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const int blk = tid + b * kAttnThreads;
        if (blk >= nblk) continue;
        const int r0 = (blk / dq) * 2, j0 = (blk % dq) * 4;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
            const int r = r0 + x;
            if (r >= R) continue;
            const int tt = r / gq, i = r - tt * gq;
            const float l = lrow[r];
#pragma unroll
            for (int y = 0; y < 4; ++y)
                put_planes(planes, plane_stride, static_cast<size_t>(t0 + tt) * ld + (g * gq + i) * d + j0 + y,
                           __fdiv_rn(acc[b][x * 4 + y], l));
        }
    }
}

// The chunk's keys / values into the ring (after the attention that reads the
// ring's older rows): positions p0 .. p0 + T - 1, of which only the last
// `capacity` survive.
__global__ void k_ring_append(const float *kc, const float *vc, int T, int p0, int KV, int d, int cap, float *k_cache,
                              float *v_cache) {
    const int first = max(0, T - cap);
    const size_t n = static_cast<size_t>(T - first) * KV * d;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(i % d);
        const size_t rest = i / d;
        const int g = static_cast<int>(rest % KV), t = first + static_cast<int>(rest / KV);
        const size_t src = (static_cast<size_t>(t) * KV + g) * d + j;
        const size_t dst = (static_cast<size_t>(g) * cap + (p0 + t) % cap) * d + j;
        k_cache[dst] = kc[src];
        v_cache[dst] = vc[src];
    }
}

// ---- GEMM on the tensor cores ----------------------------------------------------------------
// Y[m][col0 + n] (+)= sum_k X[m][k] * W[n][k] for a segment of output features,
// X given as three BF16 planes (x = x0 + x1 + x2) and W BF16 [N][K] row-major:
// three mma.sync m16n8k16 BF16 products per step, FP32 accumulation.  `resid`:
// Y = Y + scale * acc (kernels.cl:52-56), else Y = acc.
struct GemmSeg {
    const uint16_t *w;
    int n, col0, tiles;  // features, first output column, feature tiles before this segment
};
struct GemmArgs {
    const uint16_t *planes;
    size_t plane_stride;
    int lda, M, K;
    float *y;
    int ldy, resid;
    float scale;
    GemmSeg seg[3];
    int nseg;
    // grouped (tcgen05 only): grid row y < *tile_count takes tiles[y] = {group, row0, row_end}
    // and the W maps gmaps[group * nseg + segment] (global memory)
    const int4 *tiles;
    const int *tile_count;
    const CUtensorMap *gmaps;
};

__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const int bytes = valid ? 16 : 0;  // 0: zero-fill, no global read
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kGemmThreads) k_gemm_bf16x3(GemmArgs args) {
    extern __shared__ __align__(16) uint16_t gs[];
    // locate the segment of this feature tile
    int si = 0;
    while (si + 1 < args.nseg && static_cast<int>(blockIdx.x) >= args.seg[si + 1].tiles) ++si;
    const GemmSeg seg = args.seg[si];
    const int n0 = (blockIdx.x - seg.tiles) * kBN, m0 = blockIdx.y * kBM;
    const int K = args.K, ktiles = (K + kBK - 1) / kBK;
    constexpr int kStageA = 3 * kBM * kPadK, kStage = kStageA + kBN * kPadK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;  // warp tile: tokens wm*32 .. +32, features wn*16 .. +16

    auto load_stage = [&](int stage, int kt) {
        uint16_t *a = gs + stage * kStage, *b = a + kStageA;
        const int k0 = kt * kBK;
        // A: 3 planes x 64 rows x 4 chunks; B: 64 rows x 4 chunks -> 1024 chunks, 4 per thread
        for (int c = tid; c < (3 * kBM + kBN) * 4; c += kGemmThreads) {
            const int row = c >> 2, ch = c & 3, k = k0 + ch * 8;
            if (row < 3 * kBM) {
                const int pl = row / kBM, r = row - pl * kBM, m = m0 + r;
                const bool ok = m < args.M && k < K;
                const uint16_t *src = args.planes + (ok ? pl * args.plane_stride + static_cast<size_t>(m) * args.lda + k : 0);
                cp16(a + (pl * kBM + r) * kPadK + ch * 8, src, ok);
            } else {
                const int r = row - 3 * kBM, n = n0 + r;
                const bool ok = n < seg.n && k < K;
                const uint16_t *src = seg.w + (ok ? static_cast<size_t>(n) * K + k : 0);
                cp16(b + r * kPadK + ch * 8, src, ok);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // the leading part's products and the two small parts' products are summed
    // apart (each small-part term would otherwise round at the large sum's ulp)
    float acc[2][2][4], lo[2][2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = lo[i][j][e] = 0.f;

    for (int s = 0; s < kStages - 1; ++s) {
        if (s < ktiles) load_stage(s, s);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int kt = 0; kt < ktiles; ++kt) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2) : "memory");
        __syncthreads();
        const int nk = kt + kStages - 1;
        if (nk < ktiles) load_stage(nk % kStages, nk);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        const uint16_t *a = gs + (kt % kStages) * kStage, *b = a + kStageA;
#pragma unroll
        for (int ks = 0; ks < kBK; ks += 16) {
            // B fragments: features wn*16 + {0..7, 8..15}, k ks .. ks+15
            uint32_t bf[4];
            ldsm_x4(bf, b + (wn * 16 + (lane & 7) + ((lane >> 4) << 3)) * kPadK + ks + ((lane >> 3) & 1) * 8);
#pragma unroll
            for (int pl = 0; pl < 3; ++pl) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    uint32_t af[4];
                    ldsm_x4(af, a + (pl * kBM + wm * 32 + i * 16 + (lane & 15)) * kPadK + ks + (lane >> 4) * 8);
                    mma_bf16(pl == 0 ? acc[i][0] : lo[i][0], af, bf[0], bf[1]);
                    mma_bf16(pl == 0 ? acc[i][1] : lo[i][1], af, bf[2], bf[3]);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // epilogue: D rows = tokens (lane / 4, + 8), columns = features 2 (lane % 4) + {0, 1}
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = m0 + wm * 32 + i * 16 + (lane >> 2) + h * 8;
                const int n = n0 + wn * 16 + j * 8 + (lane & 3) * 2;
                if (m >= args.M) continue;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    if (n + e >= seg.n) continue;
                    float *dst = args.y + static_cast<size_t>(m) * args.ldy + seg.col0 + n + e;
                    const float v = acc[i][j][2 * h + e] + lo[i][j][2 * h + e];
                    *dst = args.resid ? __fadd_rn(*dst, __fmul_rn(args.scale, v)) : v;
                }
            }
}

// ---- GEMM on the 5th-generation tensor cores (tcgen05) ----------------------------------------
// Same product as k_gemm_bf16x3, one CTA per 128-token x BN-feature tile
// (BN 128 where that still gives a wave of CTAs, else 64: a prompt chunk has
// few 128-token tiles, and the narrower tile doubles the CTAs; the wider one
// halves the re-reads of the X planes):
// warp 0 lane 0 streams K tiles of 64 (three X planes + the W tile, 56 or 64 KB
// a stage, 128-byte swizzle) by TMA into a 3- or 4-stage ring; warp 1 lane 0 issues
// tcgen05.mma (M 128, N BN, K 16, BF16 -> FP32) into TMEM accumulators (the
// leading part, and the two small parts: summed apart as in k_gemm_bf16x3)
// and hands each stage back with tcgen05.commit; warps 2-5 read the
// accumulators (tcgen05.ld, one TMEM lane = one token row per thread) and
// apply the epilogue.  Every wait is bounded (kTcWaitNs): a wait that gives up
// sets *err and the CTA winds down.
//
// The tensor core adds each K16 step's products into its FP32 accumulator
// with one rounding of its own, so over a long K the leading part's error
// grows with K / 16 (measured: FlashLite logits 7.6e-5 from the exact values
// against the reference's own 2.0e-5).  The leading part is therefore summed
// per chunk of kLeadChunk K tiles in one of two TMEM accumulators, and the
// epilogue warps add each finished chunk into FP32 registers (round to
// nearest) while the MMAs fill the other accumulator.
constexpr int kTM = 128, kTK = 64, kTcThreads = 192;
constexpr uint32_t kTileBytes = kTM * kTK * 2;  // 16 KB: one 128 x 64 BF16 X tile
template <int BN>
constexpr uint32_t tc_stage_bytes() { return 3 * kTileBytes + BN * kTK * 2; }  // three X planes + the W tile
template <int BN>
constexpr int tc_stages() { return BN == 64 ? 4 : 3; }  // as many 56 / 64 KB stages as shared memory holds
template <int BN>
constexpr size_t tc_smem() { return 1024 + tc_stages<BN>() * tc_stage_bytes<BN>() + 256; }  // slack, tiles, barriers
constexpr unsigned long long kTcWaitNs = 2000000000ull;
constexpr int kLeadChunk = 4;  // K tiles (256 K) per leading-part accumulator chunk

struct TcMaps {
    CUtensorMap a;     // X planes: {k, token, plane}
    CUtensorMap b[3];  // W of each segment: {k, feature}
};

__device__ __forceinline__ uint64_t tc_now() { return tc::now(); }
using tc::saddr;
using tc::sw128_desc;
using tc::tmem_ld32;
__device__ __forceinline__ bool tc_try_wait(uint64_t *bar, int parity) { return tc::try_wait(bar, parity); }
__device__ __forceinline__ bool tc_wait(uint64_t *bar, int parity, int *err) { return tc::wait(bar, parity, err); }
// kind::f16 instruction descriptor: D F32, A and B BF16, both K-major, N = BN, M = 128
template <int BN>
constexpr uint32_t tc_idesc() {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
           (static_cast<uint32_t>(kTM >> 4) << 24);
}

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 1) k_gemm_tc(const __grid_constant__ TcMaps maps, GemmArgs args,
                                                           int *err) {
    constexpr uint32_t kTStageBytes = tc_stage_bytes<BN>();
    constexpr int kTStages = tc_stages<BN>();
    constexpr int kTN = BN;
    // TMEM columns: two leading-part accumulators (chunks alternate), then the small parts'
    constexpr uint32_t kTcols = BN == 128 ? 512 : 256;
    extern __shared__ uint8_t tc_raw[];
    uint8_t *tiles = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + kTStages * kTStageBytes);
    uint64_t *empty = full + kTStages, *accf = empty + kTStages;
    uint64_t *lead_full = accf + 1, *lead_empty = lead_full + 2;  // per leading accumulator
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(lead_empty + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int si = 0;
    while (si + 1 < args.nseg && static_cast<int>(blockIdx.x) >= args.seg[si + 1].tiles) ++si;
    const GemmSeg seg = args.seg[si];
    const int n0 = (blockIdx.x - seg.tiles) * kTN;
    int m0 = blockIdx.y * kTM, m_end = args.M;
    const CUtensorMap *mb = &maps.b[si];
    if (args.tiles) {  // grouped: rows and weights of this grid row's tile (unused grid rows leave at once)
        if (static_cast<int>(blockIdx.y) >= __ldg(args.tile_count)) return;
        const int4 t = __ldg(args.tiles + blockIdx.y);
        m0 = t.y;
        m_end = t.z;
        mb = args.gmaps + static_cast<size_t>(t.x) * args.nseg + si;
    }
    const int ktiles = (args.K + kTK - 1) / kTK;
    if (tid == 0) {
        for (int st = 0; st < kTStages; ++st) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&full[st])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&empty[st])) : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(accf)) : "memory");
        for (int b = 0; b < 2; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&lead_full[b])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(saddr(&lead_empty[b])) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // leading-part accumulators (columns 0..BN-1, BN..2BN-1), small parts (2BN..3BN-1)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                     "n"(kTcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    if (warp == 0 && lane == 0) {  // TMA producer
        int issued = 0;
        for (int kt = 0; kt < ktiles; ++kt) {
            const int st = kt % kTStages;
            if (kt >= kTStages && !tc_wait(&empty[st], ((kt / kTStages) - 1) & 1, err)) break;
            uint8_t *base = tiles + st * kTStageBytes;
            const uint32_t bar = saddr(&full[st]);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kTStageBytes)
                         : "memory");
            const int k0 = kt * kTK;
            for (int pl = 0; pl < 3; ++pl)
                asm volatile(
                    "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
                    "[%5];" ::"r"(saddr(base + pl * kTileBytes)),
                    "l"(&maps.a), "r"(k0), "r"(m0), "r"(pl), "r"(bar)
                    : "memory");
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                    saddr(base + 3 * kTileBytes)),
                "l"(mb), "r"(k0), "r"(n0), "r"(bar)
                : "memory");
            ++issued;
        }
        // no copy may land after the CTA has left: every issued stage is awaited (bounded)
        for (int kt = std::max(0, issued - kTStages); kt < issued; ++kt) {
            const uint64_t start = tc_now();
            while (!tc_try_wait(&full[kt % kTStages], (kt / kTStages) & 1) && tc_now() - start < kTcWaitNs) {
            }
        }
    } else if (warp == 1 && lane == 0) {  // MMA issuer
        bool ok = true;
        for (int kt = 0; kt < ktiles && ok; ++kt) {
            const int st = kt % kTStages;
            const int chunk = kt / kLeadChunk, buf = chunk & 1;
            const bool chunk_start = kt % kLeadChunk == 0;
            ok = tc_wait(&full[st], (kt / kTStages) & 1, err);
            // a leading accumulator is refilled once the epilogue has read its chunk before last
            if (ok && chunk_start && chunk >= 2) ok = tc_wait(&lead_empty[buf], ((chunk / 2) - 1) & 1, err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t base = saddr(tiles + st * kTStageBytes);
#pragma unroll
            for (int ks = 0; ks < kTK / 16; ++ks) {
                const uint64_t bd = sw128_desc(base + 3 * kTileBytes + ks * 32);
#pragma unroll
                for (int pl = 0; pl < 3; ++pl) {
                    const uint64_t ad = sw128_desc(base + pl * kTileBytes + ks * 32);
                    const uint32_t d = pl == 0 ? tmem + buf * kTN : tmem + 2 * kTN;
                    const uint32_t accumulate =
                        pl == 0 ? !(chunk_start && ks == 0) : !(kt == 0 && ks == 0 && pl == 1);
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
                        "l"(ad), "l"(bd), "r"(tc_idesc<BN>()), "r"(accumulate)
                        : "memory");
                }
            }
            // the stage is free once these MMAs have read it
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             saddr(&empty[st]))
                         : "memory");
            if (kt % kLeadChunk == kLeadChunk - 1 || kt == ktiles - 1)  // this chunk's leading sum is complete
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 saddr(&lead_full[buf]))
                             : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(accf))
                     : "memory");
    } else if (warp >= 2) {  // epilogue: thread = TMEM lane = token row of the tile
        const int quarter = warp & 3, row = quarter * 32 + lane, m = m0 + row;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const int chunks = (ktiles + kLeadChunk - 1) / kLeadChunk;
        float lead[kTN];
#pragma unroll
        for (int j = 0; j < kTN; ++j) lead[j] = 0.f;
        bool ok = true;
        for (int chunk = 0; chunk < chunks && ok; ++chunk) {  // the leading part, chunk by chunk, in order
            const int buf = chunk & 1;
            ok = __all_sync(0xffffffffu, tc_wait(&lead_full[buf], (chunk / 2) & 1, err));  // tcgen05.ld is collective
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int c = 0; c < kTN; c += 32) {
                uint32_t v[32];
                tmem_ld32(lane_base + buf * kTN + c, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) lead[c + j] = chunk ? __fadd_rn(lead[c + j], __uint_as_float(v[j]))
                                                                 : __uint_as_float(v[j]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&lead_empty[buf])) : "memory");
        }
        // every MMA has completed (also after an error: TMEM is released only then)
        const bool ready = __all_sync(0xffffffffu, tc_wait(accf, 0, err));
        if (ok && ready && ktiles > 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int c = 0; c < kTN; c += 32) {
                uint32_t v[32];
                tmem_ld32(lane_base + 2 * kTN + c, v);
                if (m < m_end) {
                    float *dst = args.y + static_cast<size_t>(m) * args.ldy + seg.col0 + n0 + c;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (n0 + c + j >= seg.n) break;
                        const float val = lead[c + j] + __uint_as_float(v[j]);
                        dst[j] = args.resid ? __fadd_rn(dst[j], __fmul_rn(args.scale, val)) : val;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTcols) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// BF16 tensor map, box 64 (K) x `rows`, 128-byte swizzle; rows past the extent read as zeros.
int encode_map(CUtensorMap *map, const void *base, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
               int rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return set_error(MR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTK), static_cast<cuuint32_t>(rows), 1u}, estride[3] = {1u, 1u, 1u};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank), const_cast<void *>(base),
                           dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(MR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return MR_OK;
}

constexpr size_t kGemmSmem = static_cast<size_t>(kStages) * (3 * kBM + kBN) * kPadK * sizeof(uint16_t);

int run_gemm(bool tcgen05, int *err, cudaStream_t stream, const uint16_t *planes, size_t plane_stride, int lda, int M,
             int K, const GemmSeg *segs, int nseg, float *y, int ldy, bool resid, float scale) {
    MR_REQUIRE(nseg >= 1 && nseg <= 3, "a batched GEMM takes 1 to 3 weight segments");
    GemmArgs a{};
    a.planes = planes;
    a.plane_stride = plane_stride;
    a.lda = lda;
    a.M = M;
    a.K = K;
    a.y = y;
    a.ldy = ldy;
    a.resid = resid ? 1 : 0;
    a.scale = scale;
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        GemmSeg t = segs[i];
        t.tiles = tiles;
        a.seg[a.nseg++] = t;
        tiles += (t.n + kBN - 1) / kBN;
    }
    if (!tcgen05) {
        const dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>((M + kBM - 1) / kBM));
        k_gemm_bf16x3<<<grid, kGemmThreads, kGemmSmem, stream>>>(a);
        MR_CUDA_TRY(cudaGetLastError());
        return MR_OK;
    }
    // tcgen05 path: 128 x 128 tiles, operands by TMA
    TcMaps maps{};
    const cuuint64_t adims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M), 3};
    const cuuint64_t astr[2] = {static_cast<cuuint64_t>(lda) * 2, static_cast<cuuint64_t>(plane_stride) * 2};
    int rc = encode_map(&maps.a, planes, 3, adims, astr, kTM);
    // 128-feature tiles when they still fill a wave of SMs, else 64
    const int mtiles = (M + kTM - 1) / kTM;
    int wide = 0;
    for (int i = 0; i < a.nseg; ++i) wide += (a.seg[i].n + 127) / 128;
    const int BN = wide * mtiles >= 148 ? 128 : 64;
    int tc_tiles = 0;
    for (int i = 0; i < a.nseg && !rc; ++i) {
        const cuuint64_t bdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(a.seg[i].n)};
        const cuuint64_t bstr[1] = {static_cast<cuuint64_t>(K) * 2};
        rc = encode_map(&maps.b[i], a.seg[i].w, 2, bdims, bstr, BN);
        a.seg[i].tiles = tc_tiles;
        tc_tiles += (a.seg[i].n + BN - 1) / BN;
    }
    if (rc) return rc;
    const dim3 grid(static_cast<unsigned>(tc_tiles), static_cast<unsigned>(mtiles));
    if (BN == 128) k_gemm_tc<128><<<grid, kTcThreads, tc_smem<128>(), stream>>>(maps, a, err);
    else k_gemm_tc<64><<<grid, kTcThreads, tc_smem<64>(), stream>>>(maps, a, err);
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

int gemm(const PrefillWork &w, cudaStream_t stream, const uint16_t *planes, size_t plane_stride, int lda, int M,
         int K, std::initializer_list<GemmSeg> segs, float *y, int ldy, bool resid, float scale) {
    return run_gemm(w.tcgen05, w.err, stream, planes, plane_stride, lda, M, K, segs.begin(), static_cast<int>(segs.size()),
                    y, ldy, resid, scale);
}

// Row width of the q | k | v buffer: FlashLighting's q | latent fits too.
int qkv_width(const PrefillModel &pm) {
    const int q = pm.heads * pm.head_dim, kv = pm.kv_max * pm.head_dim;
    return q + std::max(2 * kv, pm.lighting ? pm.latent_dim : 0);
}

size_t attn_smem(int d) {
    return sizeof(float) * (static_cast<size_t>(kAttnRows) * (d + 4) + 2 * kKT * (d + 4) +
                            2 * static_cast<size_t>(kKT) * d + kAttnRows * (kKT + 1) + 3 * kAttnRows);
}

}  // namespace

int batch_setup() {
    MR_CUDA_TRY(cudaFuncSetAttribute(k_gemm_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem<64>()));
    MR_CUDA_TRY(cudaFuncSetAttribute(k_gemm_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem<128>()));
    return MR_OK;
}

int batch_gemm(cudaStream_t stream, int *err, const uint16_t *planes, size_t plane_stride, int lda, int M, int K,
               const BatchSeg *segs, int nseg, float *y, int ldy, bool resid, float scale) {
    MR_REQUIRE(nseg >= 1 && nseg <= 3, "a batched GEMM takes 1 to 3 weight segments");
    GemmSeg g[3];
    for (int i = 0; i < nseg; ++i) g[i] = GemmSeg{static_cast<const uint16_t *>(segs[i].w), segs[i].n, segs[i].col0, 0};
    return run_gemm(true, err, stream, planes, plane_stride, lda, M, K, g, nseg, y, ldy, resid, scale);
}

int batch_weight_map(void *map, const void *w, int n, int K) {
    static_assert(sizeof(CUtensorMap) == kBatchMapBytes, "tensor map size");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(n)};
    const cuuint64_t str[1] = {static_cast<cuuint64_t>(K) * 2};
    return encode_map(static_cast<CUtensorMap *>(map), w, 2, dims, str, 128);
}

int batch_gemm_grouped(cudaStream_t stream, int *err, const uint16_t *planes, size_t plane_stride, int lda, int rows,
                       int K, const void *maps, const BatchSeg *segs, int nseg, const int *tiles,
                       const int *tile_count, int max_tiles, float *y, int ldy) {
    MR_REQUIRE(nseg >= 1 && nseg <= 3 && max_tiles > 0, "grouped GEMM arguments");
    MR_REQUIRE((reinterpret_cast<uintptr_t>(maps) & 63) == 0 && (reinterpret_cast<uintptr_t>(tiles) & 15) == 0,
               "grouped GEMM: tensor maps 64-byte and tiles 16-byte aligned");
    GemmArgs a{};
    a.planes = planes;
    a.plane_stride = plane_stride;
    a.lda = lda;
    a.M = rows;
    a.K = K;
    a.y = y;
    a.ldy = ldy;
    a.tiles = reinterpret_cast<const int4 *>(tiles);
    a.tile_count = tile_count;
    a.gmaps = static_cast<const CUtensorMap *>(maps);
    int ntiles = 0;
    for (int i = 0; i < nseg; ++i) {
        a.seg[a.nseg++] = GemmSeg{nullptr, segs[i].n, segs[i].col0, ntiles};
        ntiles += (segs[i].n + 127) / 128;
    }
    TcMaps tm{};
    const cuuint64_t adims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows), 3};
    const cuuint64_t astr[2] = {static_cast<cuuint64_t>(lda) * 2, static_cast<cuuint64_t>(plane_stride) * 2};
    if (int rc = encode_map(&tm.a, planes, 3, adims, astr, kTM)) return rc;
    const dim3 grid(static_cast<unsigned>(ntiles), static_cast<unsigned>(max_tiles));
    k_gemm_tc<128><<<grid, kTcThreads, tc_smem<128>(), stream>>>(tm, a, err);
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

int batch_rms_planes(cudaStream_t stream, const float *x, int row0, int rows, int h, int ldx, const void *gain,
                     int gain_dt, float eps, uint16_t *planes, size_t plane_stride, int ld) {
    if (rows <= 0) return MR_OK;
    k_rms_planes<<<rows, 256, 0, stream>>>(x, row0, h, ldx, gain, gain_dt, eps, planes, plane_stride, ld);
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

void prefill_release(PrefillWork &w) {
    for (void *p : {static_cast<void *>(w.x), static_cast<void *>(w.planes), static_cast<void *>(w.qkv),
                    static_cast<void *>(w.qh), static_cast<void *>(w.kc), static_cast<void *>(w.vc),
                    static_cast<void *>(w.gu), static_cast<void *>(w.logits),
                    static_cast<void *>(w.err)})
        if (p) cudaFree(p);
    const bool tc = w.tcgen05;
    w = PrefillWork{};
    w.tcgen05 = tc;
}

int prefill_reserve(const PrefillModel &pm, PrefillWork &w, int tokens, bool all_logits) {
    if (w.tokens >= tokens && (w.all_logits || !all_logits)) return MR_OK;
    const int T = std::max(tokens, w.tokens);
    const bool all = all_logits || w.all_logits;
    prefill_release(w);
    const int q = pm.heads * pm.head_dim, kv = pm.kv_max * pm.head_dim;
    w.kmax = std::max({pm.hidden, q, pm.ffn, pm.lighting ? pm.latent_dim : 0});
    auto alloc = [&](void **p, size_t bytes) -> int {
        MR_CUDA_TRY(cudaMalloc(p, bytes ? bytes : 16));
        return MR_OK;
    };
    int rc = alloc(reinterpret_cast<void **>(&w.x), sizeof(float) * T * pm.hidden);
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.planes), sizeof(uint16_t) * 3 * static_cast<size_t>(T) * w.kmax);
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.qkv), sizeof(float) * T * static_cast<size_t>(qkv_width(pm)));
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.qh), sizeof(float) * T * static_cast<size_t>(q));
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.kc), sizeof(float) * T * static_cast<size_t>(kv));
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.vc), sizeof(float) * T * static_cast<size_t>(kv));
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.gu), sizeof(float) * T * 2 * static_cast<size_t>(pm.ffn));
    if (!rc)
        rc = alloc(reinterpret_cast<void **>(&w.logits), sizeof(float) * (all ? T : 1) * static_cast<size_t>(pm.vocab));
    if (!rc) rc = alloc(reinterpret_cast<void **>(&w.err), sizeof(int));
    if (rc) {
        prefill_release(w);
        return rc;
    }
    w.tokens = T;
    w.all_logits = all;
    return MR_OK;
}

int prefill_status(const PrefillModel &pm, PrefillWork &w) {
    int err = 0;
    MR_CUDA_TRY(cudaMemcpyAsync(&err, w.err, sizeof(int), cudaMemcpyDeviceToHost, pm.stream));
    MR_CUDA_TRY(cudaStreamSynchronize(pm.stream));
    if (err) return set_error(MR_ERR_TIMEOUT, "prefill GEMM: a bounded wait gave up");
    return MR_OK;
}

int prefill_chunk(const PrefillModel &pm, PrefillWork &w, const int *d_ids, int T, int p0, bool all_logits) {
    MR_REQUIRE(T > 0 && T <= w.tokens && (!all_logits || w.all_logits), "prefill workspace too small");
    cudaStream_t st = pm.stream;
    const int h = pm.hidden, H = pm.heads, d = pm.head_dim, f = pm.ffn, q = H * d;
    const size_t ps = static_cast<size_t>(w.tokens) * w.kmax;  // plane stride
    MR_CUDA_TRY(cudaFuncSetAttribute(k_gemm_bf16x3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem));
    MR_CUDA_TRY(cudaFuncSetAttribute(k_gemm_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem<64>()));
    MR_CUDA_TRY(cudaFuncSetAttribute(k_gemm_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem<128>()));
    MR_CUDA_TRY(cudaMemsetAsync(w.err, 0, sizeof(int), st));
    MR_CUDA_TRY(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem(d)));
    k_embed_rows<<<T, 256, 0, st>>>(d_ids, T, pm.embed, pm.embed_dt, h, w.x);
    MR_CUDA_TRY(cudaGetLastError());
    for (const PrefillLayer &L : pm.layers) {
        const int KV = L.kv_heads, kv = KV * d, ldqkv = pm.lighting ? qkv_width(pm) : q + 2 * kv;
        if (pm.lighting) {
            // FlashLighting (model.py:146-190, 272-278): both branches read a_norm(x)
            const int lat = pm.latent_dim;
            k_rms_planes<<<T, 256, 0, st>>>(w.x, 0, h, h, L.a_norm, L.a_norm_dt, pm.eps, w.planes, ps, w.kmax);
            int rc = gemm(w, st, w.planes, ps, w.kmax, T, h,
                          {GemmSeg{static_cast<const uint16_t *>(L.q), q, 0, 0},
                           GemmSeg{static_cast<const uint16_t *>(L.latent), lat, q, 0}},
                          w.qkv, ldqkv, false, 0.f);
            if (!rc)
                rc = gemm(w, st, w.planes, ps, w.kmax, T, h,
                          {GemmSeg{static_cast<const uint16_t *>(L.gate), f, 0, 0},
                           GemmSeg{static_cast<const uint16_t *>(L.up), f, f, 0}},
                          w.gu, 2 * f, false, 0.f);
            if (rc) return rc;
            // k | v from latent_norm(latent), written over the latent columns
            k_rms_planes<<<T, 256, 0, st>>>(w.qkv + q, 0, lat, ldqkv, L.latent_norm, L.latent_norm_dt, pm.eps, w.planes,
                                            ps, w.kmax);
            rc = gemm(w, st, w.planes, ps, w.kmax, T, lat,
                      {GemmSeg{static_cast<const uint16_t *>(L.k), kv, q, 0},
                       GemmSeg{static_cast<const uint16_t *>(L.v), kv, q + kv, 0}},
                      w.qkv, ldqkv, false, 0.f);
            if (rc) return rc;
            const int warps = T * (H + 2 * KV);
            k_qk_rope<<<(warps * 32 + 255) / 256, 256, 0, st>>>(w.qkv, T, p0, H, KV, d, ldqkv, 1, L.q_norm, L.k_norm,
                                                                L.qk_norm_dt, pm.eps, pm.inv_freq, pm.split_half, w.qh,
                                                                w.kc, w.vc);
            MR_CUDA_TRY(cudaGetLastError());
            const int gq = H / KV, QT = std::max(1, kAttnRows / gq);
            const dim3 grid(static_cast<unsigned>((T + QT - 1) / QT), static_cast<unsigned>(KV));
            k_attention<<<grid, kAttnThreads, attn_smem(d), st>>>(w.qh, w.kc, w.vc, L.k_cache, L.v_cache, T, p0, H, KV,
                                                                  d, L.capacity, QT, w.planes, ps, w.kmax);
            MR_CUDA_TRY(cudaGetLastError());
            k_ring_append<<<256, 256, 0, st>>>(w.kc, w.vc, T, p0, KV, d, L.capacity, L.k_cache, L.v_cache);
            MR_CUDA_TRY(cudaGetLastError());
            // x += (s * attention_gate) * o, then x += (s * ffn_gate) * down (the two branches in turn)
            rc = gemm(w, st, w.planes, ps, w.kmax, T, q, {GemmSeg{static_cast<const uint16_t *>(L.o), h, 0, 0}}, w.x, h,
                      true, L.o_scale);
            if (rc) return rc;
            k_swiglu_planes<<<592, 256, 0, st>>>(w.gu, T, f, w.planes, ps, w.kmax);
            MR_CUDA_TRY(cudaGetLastError());
            rc = gemm(w, st, w.planes, ps, w.kmax, T, f, {GemmSeg{static_cast<const uint16_t *>(L.down), h, 0, 0}}, w.x,
                      h, true, L.down_scale);
            if (rc) return rc;
            continue;
        }
        // 1. RMSNorm -> q | k | v
        k_rms_planes<<<T, 256, 0, st>>>(w.x, 0, h, h, L.a_norm, L.a_norm_dt, pm.eps, w.planes, ps, w.kmax);
        int rc = gemm(w, st, w.planes, ps, w.kmax, T, h,
                      {GemmSeg{static_cast<const uint16_t *>(L.q), q, 0, 0},
                       GemmSeg{static_cast<const uint16_t *>(L.k), kv, q, 0},
                       GemmSeg{static_cast<const uint16_t *>(L.v), kv, q + kv, 0}},
                      w.qkv, ldqkv, false, 0.f);
        if (rc) return rc;
        // 2. q / k norm + RoPE; the chunk's keys and values
        {
            const int warps = T * (H + 2 * KV);
            k_qk_rope<<<(warps * 32 + 255) / 256, 256, 0, st>>>(w.qkv, T, p0, H, KV, d, ldqkv, pm.qk_norm, L.q_norm,
                                                                L.k_norm, L.qk_norm_dt, pm.eps, pm.inv_freq,
                                                                pm.split_half, w.qh, w.kc, w.vc);
            MR_CUDA_TRY(cudaGetLastError());
        }
        // 3. attention (reads the ring's older rows), then the ring append
        {
            const int gq = H / KV, QT = std::max(1, kAttnRows / gq);
            const dim3 grid(static_cast<unsigned>((T + QT - 1) / QT), static_cast<unsigned>(KV));
            k_attention<<<grid, kAttnThreads, attn_smem(d), st>>>(w.qh, w.kc, w.vc, L.k_cache, L.v_cache, T, p0, H, KV,
                                                                  d, L.capacity, QT, w.planes, ps, w.kmax);
            MR_CUDA_TRY(cudaGetLastError());
            k_ring_append<<<256, 256, 0, st>>>(w.kc, w.vc, T, p0, KV, d, L.capacity, L.k_cache, L.v_cache);
            MR_CUDA_TRY(cudaGetLastError());
        }
        // 4. o projection, x += s * o (model.py:282)
        rc = gemm(w, st, w.planes, ps, w.kmax, T, q, {GemmSeg{static_cast<const uint16_t *>(L.o), h, 0, 0}}, w.x, h, true,
                  pm.residual_scale);
        if (rc) return rc;
        // 5. RMSNorm -> gate | up -> SwiGLU -> down, x += s * down (model.py:87-89, 283)
        k_rms_planes<<<T, 256, 0, st>>>(w.x, 0, h, h, L.f_norm, L.f_norm_dt, pm.eps, w.planes, ps, w.kmax);
        rc = gemm(w, st, w.planes, ps, w.kmax, T, h,
                  {GemmSeg{static_cast<const uint16_t *>(L.gate), f, 0, 0},
                   GemmSeg{static_cast<const uint16_t *>(L.up), f, f, 0}},
                  w.gu, 2 * f, false, 0.f);
        if (rc) return rc;
        k_swiglu_planes<<<592, 256, 0, st>>>(w.gu, T, f, w.planes, ps, w.kmax);
        MR_CUDA_TRY(cudaGetLastError());
        rc = gemm(w, st, w.planes, ps, w.kmax, T, f, {GemmSeg{static_cast<const uint16_t *>(L.down), h, 0, 0}}, w.x, h,
                  true, pm.residual_scale);
        if (rc) return rc;
    }
    // final RMSNorm + lm_head for the rows whose logits are wanted (model.py:285, 307)
    const int r0 = all_logits ? 0 : T - 1, rows = all_logits ? T : 1;
    k_rms_planes<<<rows, 256, 0, st>>>(w.x, r0, h, h, pm.final_norm, pm.final_norm_dt, pm.eps, w.planes, ps, w.kmax);
    return gemm(w, st, w.planes, ps, w.kmax, rows, h, {GemmSeg{static_cast<const uint16_t *>(pm.head), pm.vocab, 0, 0}},
                w.logits, pm.vocab, false, 0.f);
}

}  // namespace mr
