// Heavy Medium sparse attention in one launch (included by heavy.cu only):
// model.py:192-229 from the q / latent projections to the attended vector.
//
// Grid: KV heads x (chunks + 1) units of 256 threads.  Unit u < chunks of KV
// head kh ("window unit") attends the window keys [u*CH, (u+1)*CH) that
// earlier tokens wrote (every window key but the newest) for the G = H / KVH
// query heads of kh, after computing its share of kh's rows of
// kv = W_kv_up latent and counting them in ready[kh]; no window unit waits for
// anything but the previous kernel.  Each leaves a partial softmax (max, sum,
// weighted values) per query head and counts itself in wdone[kh].  Unit
// `chunks` ("block unit") scores and ranks the full blocks (which the new row
// cannot change) and gathers the best ones' mean values first; then it waits
// for ready[kh], appends the new row, forms its own partial over the kept
// blocks and the newest key, waits for wdone[kh] and merges the window units'
// partials and its own into the output (all their loads in one round).
//
// Arithmetic: q / k non-affine RMSNorm (eps 1e-6) + RoPE in float32 with the
// reference's roundings; block means as kernels.cl block_means' running sum
// (kept incrementally: a full block's sum never changes, so the newest block's
// running sum is carried from token to token and gives the same bits as the
// loop); the distance penalty and the stable top-k as model.py:220-226 (ties
// to the lower block).  Scores are float32 dot products (one thread per score,
// FMA in column order) and the softmax over window and kept blocks is merged
// from partials, so kept blocks agree with the reference's except where its
// own scores tie within rounding, and attended values within the parity
// tolerance.
//
// Before its dependency wait every unit asks L2 for what it will read that no
// kernel in flight writes: its kv_up rows, its window rows of the ring
// (written by earlier tokens), the full blocks' means.
#pragma once

namespace attn {

constexpr int kThreads = 256;
constexpr int kChunk = 64;      // window keys per unit
constexpr int kPad = kChunk + 1;  // transposed tile row: column t of key row j at j * kPad + t (no bank conflict)
constexpr int kMaxG = 8;        // query heads per KV head
constexpr int kMaxDim = 128;
// registers per thread: at most 144, so that a streaming CTA of the next kernel (9 warps of
// <= 96 registers) fits beside a unit on the SM's 64 K registers (7.654 against 7.666 ms per
// heavy-medium-2.0 token)
constexpr int kMaxRegs = 144;
constexpr int kMergeBatch = 16;  // window units merged from registers in one load round (more: loaded as used)

struct Args {
    const float *q;                      // [H * d] raw queries
    const float *latent;                 // [latent_dim]
    const void *kv_up;                   // [2 * width, latent_dim]
    int kv_dtype, latent_dim;
    float *kv;                           // [2 * width] raw keys | values of this token
    float *k_ring, *v_ring;              // [context][width]
    float *k_mean, *v_mean;              // [max blocks][width]
    float *k_bsum, *v_bsum;              // [width]: running sums of the newest block
    const float *inv_freq;
    int split_half;
    int H, KVH, d, position, count, length, start, blocks, block, slots, slots_max, chunks, max_blocks;
    const float *log1p_table;
    float slope;
    int *kept;                           // [H][slots_max]
    float *partial;                      // [KVH][chunks + 1][G][d + 2]: the window units' partials
    unsigned long long *ready, *wdone;   // [KVH] monotonic counters (targets seq * chunks)
    unsigned long long seq;              // this launch's number (1, 2, ...)
    float *out;                          // [H * d]
    int *err;
    unsigned long long *probe;           // tracing only (heavy.cu probe), else NULL
    unsigned long long wait_ns;          // how long the key / value wait may last
    int withhold;                        // fault injection: the units do not count their rows
};

__device__ __forceinline__ bool wait_count(const unsigned long long *c, unsigned long long target, int *err,
                                           uint64_t limit) {
    const uint64_t start = global_time_ns();
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if (*reinterpret_cast<volatile int *>(err)) return false;  // another wait already gave up
        if (global_time_ns() - start > limit) {
            atomicCAS(err, 0, 3);
            return false;
        }
        __nanosleep(64);
    }
}

// One warp: non-affine RMSNorm (eps 1e-6) then RoPE at `position` of one head
// (d values at src), written to dst.
__device__ __forceinline__ void norm_rope(const float *src, float *dst, int dim, int split_half, int position,
                                          const float *inv_freq) {
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
#pragma unroll 4
    for (int j = lane; j < dim; j += 32) ss = fmaf(src[j], src[j], ss);
    ss = warp_sum(ss);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(FADD(__fdiv_rn(ss, static_cast<float>(dim)), 1e-6f)));
    const int half = dim / 2;
    float u[4], v[4];
    int n = 0;
    for (int p = lane; p < half && n < 4; p += 32, ++n) {
        const int j = split_half ? p : 2 * p, k = split_half ? p + half : 2 * p + 1;
        u[n] = FMUL(src[j], scale);
        v[n] = FMUL(src[k], scale);
    }
    __syncwarp();
    n = 0;
    for (int p = lane; p < half && n < 4; p += 32, ++n) {
        const int j = split_half ? p : 2 * p, k = split_half ? p + half : 2 * p + 1;
        const float angle = FMUL(static_cast<float>(position), inv_freq[p]);
        float s, c;
        sincosf(angle, &s, &c);
        dst[j] = __fsub_rn(FMUL(u[n], c), FMUL(v[n], s));
        dst[k] = FADD(FMUL(u[n], s), FMUL(v[n], c));
    }
    __syncwarp();
}

// n (<= kChunk) rows [row0, row0 + n) of a [*, width] float matrix, columns
// [col, col + d): keys transposed into kT (column t of row j at j * kPad + t)
// and, when vt is given, the same rows of `vsrc` row-major into vt (n x d).
// Relative row `fresh_at` comes from kfresh / vfresh instead.  The loads
// (Tile::load) and the stores (Tile::store) are separate calls, so that other
// work can run while the loads are in flight.
struct Tile {
    static constexpr int kPer = kChunk * kMaxDim / 4 / kThreads;
    float4 kv[kPer], vv[kPer];
    __device__ __forceinline__ void load(const float *ksrc, const float *vsrc, size_t row0, int width, int col, int n,
                                         int d, int fresh_at, const float *kfresh, const float *vfresh) {
        const int q = d / 4, total = n * q;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kThreads, t = i / q, c = i % q;
            const size_t at = (row0 + t) * width + col;
            kv[k] = i >= total    ? float4{}
                    : t == fresh_at ? reinterpret_cast<const float4 *>(kfresh)[c]
                                    : __ldcg(reinterpret_cast<const float4 *>(ksrc + at) + c);
            vv[k] = (i >= total || !vsrc) ? float4{}
                    : t == fresh_at       ? reinterpret_cast<const float4 *>(vfresh)[c]
                                          : __ldcg(reinterpret_cast<const float4 *>(vsrc + at) + c);
        }
    }
    __device__ __forceinline__ void store(float *kT, float *vt, int n, int d) const {
        const int q = d / 4, total = n * q;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kThreads, t = i / q, c = i % q;
            if (i >= total) continue;
            kT[(4 * c) * kPad + t] = kv[k].x;
            kT[(4 * c + 1) * kPad + t] = kv[k].y;
            kT[(4 * c + 2) * kPad + t] = kv[k].z;
            kT[(4 * c + 3) * kPad + t] = kv[k].w;
            if (vt) reinterpret_cast<float4 *>(vt + t * d)[c] = vv[k];
        }
    }
};
__device__ __forceinline__ void load_tile(float *kT, float *vt, const float *ksrc, const float *vsrc, size_t row0,
                                          int width, int col, int n, int d, int fresh_at, const float *kfresh,
                                          const float *vfresh) {
    Tile tile;
    tile.load(ksrc, vt ? vsrc : nullptr, row0, width, col, n, d, fresh_at, kfresh, vfresh);
    tile.store(kT, vt, n, d);
}

// q . (column t of kT) / sqrt(d): one thread, columns in order, four FMA chains.
__device__ __forceinline__ float tile_score(const float *qh, const float *kT, int t, int d) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
    for (int j = 0; j < d; j += 4) {
        const float4 q4 = *reinterpret_cast<const float4 *>(qh + j);  // one broadcast load for four columns
        a0 = fmaf(q4.x, kT[j * kPad + t], a0);
        a1 = fmaf(q4.y, kT[(j + 1) * kPad + t], a1);
        a2 = fmaf(q4.z, kT[(j + 2) * kPad + t], a2);
        a3 = fmaf(q4.w, kT[(j + 3) * kPad + t], a3);
    }
    return __fdiv_rn((a0 + a1) + (a2 + a3), __fsqrt_rn(static_cast<float>(d)));
}

// L2 prefetch of n rows of d floats, `stride` floats apart (one row per thread).
__device__ __forceinline__ void prefetch_rows(const float *first, size_t stride, int n, int d) {
    for (int t = threadIdx.x; t < n; t += kThreads) prefetch_l2(first + t * stride, d * sizeof(float));
}


// q . k / sqrt(d) for one contiguous key row (both 16-byte aligned in shared
// memory), tile_score's arithmetic; the loads run ahead of the four FMA chains.
__device__ __forceinline__ float row_score(const float *qh, const float *k, int d) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 8
    for (int j = 0; j < d; j += 4) {
        const float4 q4 = *reinterpret_cast<const float4 *>(qh + j), k4 = *reinterpret_cast<const float4 *>(k + j);
        a0 = fmaf(q4.x, k4.x, a0);
        a1 = fmaf(q4.y, k4.y, a1);
        a2 = fmaf(q4.z, k4.z, a2);
        a3 = fmaf(q4.w, k4.w, a3);
    }
    return __fdiv_rn((a0 + a1) + (a2 + a3), __fsqrt_rn(static_cast<float>(d)));
}

// Shared memory of one unit, in floats (ints take a float's place).
struct Smem {
    float *lat, *qs, *knew, *vnew, *kmean, *vmean, *kT, *vt, *ps, *bscore, *pen, *bpart, *wts, *sk, *sb, *ml;
    int *cnt, *joins, *top, *kept_s, *row_s;
    __device__ __host__ static size_t floats(int latent_dim, int G, int d, int max_blocks, int slots_max, int chunks) {
        return ((latent_dim + 3) & ~3) + static_cast<size_t>(G) * d + 4 * static_cast<size_t>(d) +
               ((static_cast<size_t>(d) * kPad + 3) & ~static_cast<size_t>(3)) + static_cast<size_t>(kChunk) * d +
               static_cast<size_t>(G) * kChunk + static_cast<size_t>(G) * max_blocks + max_blocks +
               static_cast<size_t>(G) * (d + 2) + static_cast<size_t>(G) * (slots_max + 1) + 4 * static_cast<size_t>(G) +
               2 * static_cast<size_t>(chunks) * G + static_cast<size_t>(G) * slots_max +
               2 * static_cast<size_t>(G) * (slots_max + 1);
    }
    __device__ Smem(float *sm, const Args &a, int G) {
        const int d = a.d;
        lat = sm;
        qs = lat + ((a.latent_dim + 3) & ~3);
        knew = qs + G * d;       // the new row: key (normalised, rotated) and value
        vnew = knew + d;
        kmean = vnew + d;        // the newest block's mean key / value
        vmean = kmean + d;
        kT = vmean + d;          // [d][kPad]
        vt = kT + ((d * kPad + 3) & ~3);  // [kChunk][d]; block unit: [G][slots_max][d] kept mean values
        ps = vt + kChunk * d;    // [G][kChunk]
        bscore = ps + G * kChunk;         // block unit: [G][max_blocks]
        pen = bscore + G * a.max_blocks;  // [max_blocks]
        bpart = pen + a.max_blocks;       // block unit: [G][d + 2] its partial
        wts = bpart + G * (d + 2);        // [G][slots_max + 1] softmax weights
        sk = wts + G * (a.slots_max + 1);  // [G] the newest key's score
        sb = sk + G;                        // [G] the newest block's score
        ml = sb + G;                        // merge: [chunks][G][2]
        cnt = reinterpret_cast<int *>(ml + 2 * a.chunks * G);  // [G] kept full blocks
        joins = cnt + G;                    // [G] the newest block is kept
        top = joins + G;                    // [G][slots_max] best full blocks, best first
        kept_s = top + G * a.slots_max;     // [G][slots_max + 1] kept ids ascending
        row_s = kept_s + G * (a.slots_max + 1);  // [G][slots_max + 1] their rows of vt
    }
};

// Window unit: kv rows, queries, the window partial of keys [t0, t0 + n).
__device__ void window_unit(const Args &a, const Smem &s, int kh, int u, int G) {
    const int d = a.d, width = a.KVH * d, units = a.chunks + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kThreads / 32;
    const int t0 = u * kChunk, n = max(0, min(kChunk, a.length - 1 - t0));
    const int r0 = 2 * d * u / a.chunks, r1 = 2 * d * (u + 1) / a.chunks;
    const size_t lrow = static_cast<size_t>(a.latent_dim) * (a.kv_dtype == MR_DTYPE_F32 ? 4 : 2);
    // 1. the latent and the group's queries in one load round; this unit's rows
    //    of kv = W_kv_up latent (keys kh*d .., values width + kh*d ..)
    //    (the window tile's loads, which need nothing of this token, go out first)
    Tile tile;
    tile.load(a.k_ring, a.v_ring, static_cast<size_t>(a.start + t0), width, kh * d, n, d, -1, nullptr, nullptr);
    for (int i = threadIdx.x; i < a.latent_dim; i += kThreads) s.lat[i] = __ldcg(a.latent + i);
    for (int i = threadIdx.x; i < G * d; i += kThreads) s.qs[i] = __ldcg(a.q + static_cast<size_t>(kh) * G * d + i);
    __syncthreads();
    for (int r = r0 + warp; r < r1; r += nwarps) {
        const int row = r < d ? kh * d + r : width + kh * d + (r - d);
        const char *rp = static_cast<const char *>(a.kv_up) + row * lrow;
        float acc = 0.f;
        if ((lrow & 15) == 0) {
            const int per = a.kv_dtype == MR_DTYPE_F32 ? 4 : 8, nv = a.latent_dim / per;
            constexpr int kIn = 8;  // 16-byte chunks per lane in flight (a 512-wide BF16 row is 2)
            for (int c0 = lane; c0 < nv; c0 += 32 * kIn) {
                uint4 w[kIn];
#pragma unroll
                for (int k = 0; k < kIn; ++k)
                    w[k] = c0 + 32 * k < nv ? __ldg(reinterpret_cast<const uint4 *>(rp) + c0 + 32 * k) : uint4{};
#pragma unroll
                for (int k = 0; k < kIn; ++k)
                    if (c0 + 32 * k < nv) acc += dot16(w[k], s.lat + per * (c0 + 32 * k), a.kv_dtype);
            }
        } else {
            for (int j = lane; j < a.latent_dim; j += 32) acc = fmaf(load_weight(rp, a.kv_dtype, j), s.lat[j], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) a.kv[row] = acc;
    }
    __threadfence();  // each writer's rows are visible device-wide before the count goes up
    __syncthreads();
    if (threadIdx.x == 0) {
        if (!a.withhold) atomicAdd(&a.ready[kh], 1ull);
        probe(a.probe, kProbeStaged);
    }
    // 2. the queries normalised and rotated; the window keys and values
    for (int g = warp; g < G; g += nwarps) norm_rope(s.qs + g * d, s.qs + g * d, d, a.split_half, a.position, a.inv_freq);
    tile.store(s.kT, s.vt, n, d);
    __syncthreads();
    float *part = a.partial + (static_cast<size_t>(kh) * units + u) * G * (d + 2);
    for (int i = threadIdx.x; i < G * n; i += kThreads) {
        const int g = i / n, t = i % n;
        s.ps[g * kChunk + t] = tile_score(s.qs + g * d, s.kT, t, d);
    }
    __syncthreads();
    if (threadIdx.x == 0) probe(a.probe, kProbeX5);  // window units: scores done
    // per query head: max, exp and sum (warp g), then the value mix
    for (int g = warp; g < G; g += nwarps) {
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, s.ps[g * kChunk + t]);
        m = warp_max(m);
        float l = 0.f;
        for (int t = lane; t < n; t += 32) {
            const float e = expf(__fsub_rn(s.ps[g * kChunk + t], m));
            s.ps[g * kChunk + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            part[g * (d + 2) + d] = n ? m : -INFINITY;
            part[g * (d + 2) + d + 1] = n ? l : 0.f;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * d; i += kThreads) {
        const int g = i / d, j = i % d;
        float acc = 0.f;
        int t = 0;
        for (; t + 4 <= n; t += 4) {  // four weights in one broadcast load
            const float4 p4 = *reinterpret_cast<const float4 *>(s.ps + g * kChunk + t);
            acc = fmaf(p4.x, s.vt[t * d + j], acc);
            acc = fmaf(p4.y, s.vt[(t + 1) * d + j], acc);
            acc = fmaf(p4.z, s.vt[(t + 2) * d + j], acc);
            acc = fmaf(p4.w, s.vt[(t + 3) * d + j], acc);
        }
        for (; t < n; ++t) acc = fmaf(s.ps[g * kChunk + t], s.vt[t * d + j], acc);
        part[g * (d + 2) + j] = acc;
    }
    // 3. counted once its partial is visible
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        atomicAdd(&a.wdone[kh], 1ull);
        probe(a.probe, kProbeMain);
    }
}

// Block unit: the full blocks' scores and ranks and the best ones' mean values
// (no dependency on the new row), then the new row, the newest block, the kept
// list, this unit's partial and the merge of every unit's partial.
__device__ void block_unit(const Args &a, const Smem &s, int kh, int G) {
    const int d = a.d, width = a.KVH * d, units = a.chunks + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kThreads / 32;
    const int b = a.blocks - 1;             // the newest block; 0 .. b-1 are full and fixed
    const int nold = min(a.slots, b);       // full blocks that can be kept
    const int first = (a.count - 1) % a.block == 0;
    const int SM = a.slots_max;
    __shared__ int stop;  // one thread's reading, so that every thread takes the same branch
    // 1. queries; distance penalties (model.py:220-222); the newest block's running sums
    for (int i = threadIdx.x; i < G * d; i += kThreads) s.qs[i] = __ldcg(a.q + static_cast<size_t>(kh) * G * d + i);
    for (int bb = threadIdx.x; bb < a.blocks; bb += kThreads)
        s.pen[bb] = FMUL(a.slope, a.log1p_table[a.position - min((bb + 1) * a.block - 1, a.position)]);
    for (int i = threadIdx.x; i < G * SM; i += kThreads) s.top[i] = 0;  // in range whatever the scores
    float ksum = 0.f, vsum = 0.f;
    if (threadIdx.x < d && !first) {
        ksum = __ldcg(a.k_bsum + kh * d + threadIdx.x);
        vsum = __ldcg(a.v_bsum + kh * d + threadIdx.x);
    }
    __syncthreads();
    for (int g = warp; g < G; g += nwarps) norm_rope(s.qs + g * d, s.qs + g * d, d, a.split_half, a.position, a.inv_freq);
    // 2. scores of the full blocks minus the penalty, kChunk mean keys at a time
    for (int b0 = 0; b0 < b; b0 += kChunk) {
        const int nb = min(kChunk, b - b0);
        __syncthreads();
        load_tile(s.kT, nullptr, a.k_mean, nullptr, static_cast<size_t>(b0), width, kh * d, nb, d, -1, nullptr,
                  nullptr);
        __syncthreads();
        for (int i = threadIdx.x; i < G * nb; i += kThreads) {
            const int g = i / nb, t = i % nb;
            s.bscore[g * a.max_blocks + b0 + t] = __fsub_rn(tile_score(s.qs + g * d, s.kT, t, d), s.pen[b0 + t]);
        }
    }
    __syncthreads();
    // 3. the best `nold` full blocks per head, best first (stable: ties to the lower block)
    for (int i = threadIdx.x; i < G * b; i += kThreads) {
        const int g = i / b, bb = i % b;
        const float *sc = s.bscore + g * a.max_blocks;
        const float v = sc[bb];
        int r = 0;
        for (int j = 0; j < b; ++j) r += (sc[j] > v) || (sc[j] == v && j < bb);
        if (r < nold) s.top[g * SM + r] = bb;
    }
    __syncthreads();
    // 4. their mean values into rows [g][r] of vt, all loads before the first store
    {
        constexpr int kPer = kChunk * kMaxDim / 4 / kThreads;
        const int q4 = d / 4, total = G * nold * q4, nd = max(nold, 1);
        float4 v[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kThreads, gr = i / q4, c = i % q4;
            v[k] = i < total ? __ldcg(reinterpret_cast<const float4 *>(
                                          a.v_mean + static_cast<size_t>(s.top[(gr / nd) * SM + gr % nd]) * width +
                                          kh * d) + c)
                             : float4{};
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kThreads, gr = i / q4, c = i % q4;
            if (i < total) reinterpret_cast<float4 *>(s.vt + ((gr / nd) * SM + gr % nd) * d)[c] = v[k];
        }
    }
    // 5. the new key / value
    if (threadIdx.x == 0) stop = !wait_count(&a.ready[kh], a.seq * a.chunks, a.err, a.wait_ns);
    __syncthreads();
    if (stop) return;
    for (int j = threadIdx.x; j < d; j += kThreads) {
        s.knew[j] = __ldcg(a.kv + kh * d + j);
        s.vnew[j] = __ldcg(a.kv + width + kh * d + j);
    }
    __syncthreads();
    if (warp == 0) norm_rope(s.knew, s.knew, d, a.split_half, a.position, a.inv_freq);
    __syncthreads();
    if (threadIdx.x == 0) probe(a.probe, kProbeX6);
    // 6. append the row; the newest block's running sums and mean (kernels.cl block_means)
    {
        const float inv_n = static_cast<float>(a.count - b * a.block);
        const size_t row = static_cast<size_t>(a.count - 1);
        for (int j = threadIdx.x; j < d; j += kThreads) {
            const size_t at = static_cast<size_t>(kh) * d + j;
            a.k_ring[row * width + at] = s.knew[j];
            a.v_ring[row * width + at] = s.vnew[j];
            const float ks = first ? FADD(0.f, s.knew[j]) : FADD(ksum, s.knew[j]);
            const float vs = first ? FADD(0.f, s.vnew[j]) : FADD(vsum, s.vnew[j]);
            a.k_bsum[at] = ks;
            a.v_bsum[at] = vs;
            s.kmean[j] = __fdiv_rn(ks, inv_n);
            s.vmean[j] = __fdiv_rn(vs, inv_n);
            a.k_mean[static_cast<size_t>(b) * width + at] = s.kmean[j];
            a.v_mean[static_cast<size_t>(b) * width + at] = s.vmean[j];
        }
    }
    __syncthreads();
    // 7. scores of the newest key (threads 0..G-1) and the newest block (G..2G-1)
    if (threadIdx.x < 2 * G) {
        const int g = threadIdx.x % G;
        if (threadIdx.x < G) {
            s.sk[g] = row_score(s.qs + g * d, s.knew, d);
        } else {
            const float v = __fsub_rn(row_score(s.qs + g * d, s.kmean, d), s.pen[b]);
            s.sb[g] = v;
            s.bscore[g * a.max_blocks + b] = v;
        }
    }
    __syncthreads();
    // 8. kept blocks: the newest joins when it beats the last of the best `slots` full
    //    blocks (a tie keeps the lower block), pushing that one out; -inf scores drop
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        const float *sc = s.bscore + g * a.max_blocks;
        const float snew = s.sb[g];
        const bool joins = snew != -INFINITY && (nold < a.slots || (nold > 0 && snew > sc[s.top[g * SM + nold - 1]]));
        int kn = joins && nold == a.slots ? nold - 1 : nold;
        while (kn > 0 && sc[s.top[g * SM + kn - 1]] == -INFINITY) --kn;
        s.cnt[g] = kn;
        s.joins[g] = joins;
        if (joins) {  // the newest block (the largest id: last in ascending order) in row kn of vt
            s.kept_s[g * (SM + 1) + kn] = b;
            s.row_s[g * (SM + 1) + kn] = kn;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * SM; i += kThreads) {  // the full ones in ascending order
        const int g = i / SM, r = i % SM;
        if (r < s.cnt[g]) {
            const int id = s.top[g * SM + r];
            int pos = 0;
            for (int r2 = 0; r2 < s.cnt[g]; ++r2) pos += s.top[g * SM + r2] < id;
            s.kept_s[g * (SM + 1) + pos] = id;
            s.row_s[g * (SM + 1) + pos] = r;
        }
    }
    for (int i = threadIdx.x; i < G * d; i += kThreads) {  // the newest block's mean value in row cnt[g]
        const int g = i / d, j = i % d;
        if (s.joins[g]) s.vt[(g * SM + s.cnt[g]) * d + j] = s.vmean[j];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * SM; i += kThreads) {  // the kept ids per head, -1 padded
        const int g = i / SM, k = i % SM;
        const int nk = s.cnt[g] + s.joins[g];
        a.kept[(kh * G + g) * SM + k] = k < nk ? s.kept_s[g * (SM + 1) + k] : -1;
    }
    // 9. this unit's partial per head (warp g): the kept blocks, then the newest key
    for (int g = warp; g < G; g += nwarps) {
        const int nk = s.cnt[g] + s.joins[g];
        const float *sc = s.bscore + g * a.max_blocks;
        const int *ks = s.kept_s + g * (SM + 1);
        float *w = s.wts + g * (SM + 1);
        float m = -INFINITY;
        for (int e = lane; e <= nk; e += 32) m = fmaxf(m, e < nk ? sc[ks[e]] : s.sk[g]);
        m = warp_max(m);
        float l = 0.f;
        for (int e = lane; e <= nk; e += 32) {
            const float x = expf(__fsub_rn(e < nk ? sc[ks[e]] : s.sk[g], m));
            w[e] = x;
            l += x;
        }
        l = warp_sum(l);
        __syncwarp();
        // columns lane, lane + 32, ... (d <= kMaxDim); each column's sum in kept order
        const int *rows = s.row_s + g * (SM + 1);
        constexpr int kCols = kMaxDim / 32;
        float acc[kCols] = {};
        for (int e = 0; e < nk; ++e) {
            const float we = w[e];
            const float *v = s.vt + (g * SM + rows[e]) * d;
#pragma unroll
            for (int q = 0; q < kCols; ++q)
                if (lane + 32 * q < d) acc[q] = fmaf(we, v[lane + 32 * q], acc[q]);
        }
#pragma unroll
        for (int q = 0; q < kCols; ++q)
            if (lane + 32 * q < d) s.bpart[g * (d + 2) + lane + 32 * q] = fmaf(w[nk], s.vnew[lane + 32 * q], acc[q]);
        if (lane == 0) {
            s.bpart[g * (d + 2) + d] = m;
            s.bpart[g * (d + 2) + d + 1] = l;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        probe(a.probe, kProbeX7);
        stop = !wait_count(&a.wdone[kh], a.seq * a.chunks, a.err, a.wait_ns);
    }
    __syncthreads();
    if (stop) return;
    // 10. the window units' partials (in unit order) and this unit's, merged: every unit's
    //     max and sum staged and this thread's weighted values loaded in one round
    const float *base = a.partial + static_cast<size_t>(kh) * units * G * (d + 2);
    for (int i = threadIdx.x; i < a.chunks * G; i += kThreads) {
        s.ml[2 * i] = __ldcg(base + i * (d + 2) + d);
        s.ml[2 * i + 1] = __ldcg(base + i * (d + 2) + d + 1);
    }
    const bool one_round = G * d <= 2 * kThreads && a.chunks <= kMergeBatch;
    float acc[2][kMergeBatch];
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int i = threadIdx.x + it * kThreads, g = i / d, j = i % d;
#pragma unroll
        for (int k = 0; k < kMergeBatch; ++k)
            acc[it][k] = one_round && i < G * d && k < a.chunks ? __ldcg(base + (k * G + g) * (d + 2) + j) : 0.f;
    }
    __syncthreads();
    // item i = (head g, column j): the maximum over every unit, then the window units in
    // order and this unit last, each scaled by exp(its max - the maximum)
    auto maximum = [&](int g) {
        float mx = s.bpart[g * (d + 2) + d];
        for (int v = 0; v < a.chunks; ++v) mx = fmaxf(mx, s.ml[2 * (v * G + g)]);
        return mx;
    };
    auto finish = [&](int i, float num, float den, float mx) {
        const int g = i / d, j = i % d;
        const float mb = s.bpart[g * (d + 2) + d];
        if (mb != -INFINITY) {
            const float f = expf(__fsub_rn(mb, mx));
            num = fmaf(s.bpart[g * (d + 2) + j], f, num);
            den = fmaf(s.bpart[g * (d + 2) + d + 1], f, den);
        }
        a.out[static_cast<size_t>(kh * G + g) * d + j] = __fdiv_rn(num, den);
    };
    if (one_round) {
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const int i = threadIdx.x + it * kThreads, g = i / d;
            if (i >= G * d) break;
            const float mx = maximum(g);
            float num = 0.f, den = 0.f;
#pragma unroll
            for (int k = 0; k < kMergeBatch; ++k) {
                if (k >= a.chunks) break;
                const float mv = s.ml[2 * (k * G + g)];
                if (mv == -INFINITY) continue;
                const float f = expf(__fsub_rn(mv, mx));
                num = fmaf(acc[it][k], f, num);
                den = fmaf(s.ml[2 * (k * G + g) + 1], f, den);
            }
            finish(i, num, den, mx);
        }
    } else {
        for (int i = threadIdx.x; i < G * d; i += kThreads) {
            const int g = i / d, j = i % d;
            const float mx = maximum(g);
            float num = 0.f, den = 0.f;
            for (int v = 0; v < a.chunks; ++v) {
                const float mv = s.ml[2 * (v * G + g)];
                if (mv == -INFINITY) continue;
                const float f = expf(__fsub_rn(mv, mx));
                num = fmaf(__ldcg(base + (v * G + g) * (d + 2) + j), f, num);
                den = fmaf(s.ml[2 * (v * G + g) + 1], f, den);
            }
            finish(i, num, den, mx);
        }
    }
}

__global__ void __maxnreg__(kMaxRegs) k_sparse_attention(Args a) {
    pdl_trigger();
    extern __shared__ __align__(16) float sm[];
    const int units = a.chunks + 1;
    const int kh = blockIdx.x / units, u = blockIdx.x % units;
    const int G = a.H / a.KVH, d = a.d, width = a.KVH * d;
    const Smem s(sm, a, G);
    const bool block = u == a.chunks;
    // 0. before the wait: L2 prefetch of what this unit reads that no kernel in flight writes
    if (!block) {
        const int r0 = 2 * d * u / a.chunks, r1 = 2 * d * (u + 1) / a.chunks;
        const size_t lrow = static_cast<size_t>(a.latent_dim) * (a.kv_dtype == MR_DTYPE_F32 ? 4 : 2);
        const int t0 = u * kChunk, n = max(0, min(kChunk, a.length - 1 - t0));
        if (threadIdx.x == 0) {
            const char *base = static_cast<const char *>(a.kv_up);
            if (r0 < min(r1, d)) prefetch_l2(base + (kh * d + r0) * lrow, (min(r1, d) - r0) * lrow);
            if (max(r0, d) < r1)
                prefetch_l2(base + (width + kh * d + max(r0, d) - d) * lrow, (r1 - max(r0, d)) * lrow);
        }
        prefetch_rows(a.k_ring + static_cast<size_t>(a.start + t0) * width + kh * d, width, n, d);
        prefetch_rows(a.v_ring + static_cast<size_t>(a.start + t0) * width + kh * d, width, n, d);
    } else {
        prefetch_rows(a.k_mean + kh * d, width, a.blocks - 1, d);
        prefetch_rows(a.v_mean + kh * d, width, a.blocks - 1, d);
    }
    if (threadIdx.x == 0) probe(a.probe, kProbeStart);
    pdl_wait();
    if (threadIdx.x == 0) probe(a.probe, kProbeWaited);
    if (block) {
        block_unit(a, s, kh, G);
        __syncthreads();
        if (threadIdx.x == 0) probe(a.probe, kProbeExit);
    } else {
        window_unit(a, s, kh, u, G);
    }
}

// Shared memory of one unit (bytes): Smem's regions.
inline size_t smem_bytes(int latent_dim, int G, int d, int max_blocks, int slots_max, int chunks) {
    return Smem::floats(latent_dim, G, d, max_blocks, slots_max, chunks) * sizeof(float);
}

}  // namespace attn
