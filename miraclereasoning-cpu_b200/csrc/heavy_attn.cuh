// Heavy Medium sparse attention in one launch (included by heavy.cu only):
// model.py:192-229 from the q / latent projections to the attended vector.
//
// Grid: KV heads x (chunks + 1) units of 256 threads.  Unit u < chunks of KV
// head kh attends window keys [u*CH, (u+1)*CH) for the G = H / KVH query heads
// of kh; unit `chunks` is the head's block unit (block means, block scores,
// top-k, kept blocks).  Every unit first computes its share of kh's rows of
// kv = W_kv_up latent and counts them in ready[kh]; only the units that need
// the new key / value (the block unit and the window unit holding the newest
// row) wait for that count.  Each unit leaves a partial softmax (max, sum,
// weighted values) per query head; the last unit of kh to finish merges them.
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
// (written by earlier tokens), the block means.
#pragma once

namespace attn {

constexpr int kThreads = 256;
constexpr int kChunk = 64;      // window keys per unit
constexpr int kPad = kChunk + 1;  // transposed tile row: column t of key row j at j * kPad + t (no bank conflict)
constexpr int kMaxG = 8;        // query heads per KV head
constexpr int kMaxDim = 128;
constexpr int kMergeBatch = 32;

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
    float *partial;                      // [KVH][chunks + 1][G][d + 2]
    unsigned long long *ready, *done;    // [KVH] monotonic counters
    unsigned long long seq;              // this launch's number (1, 2, ...): targets seq * units
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
// Relative row `fresh_at` comes from kfresh / vfresh instead.  Every load is
// issued before the first store.
__device__ __forceinline__ void load_tile(float *kT, float *vt, const float *ksrc, const float *vsrc, size_t row0,
                                          int width, int col, int n, int d, int fresh_at, const float *kfresh,
                                          const float *vfresh) {
    constexpr int kPer = kChunk * kMaxDim / 4 / kThreads;
    const int q = d / 4, total = n * q;
    float4 kv[kPer], vv[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = threadIdx.x + k * kThreads, t = i / q, c = i % q;
        const size_t at = (row0 + t) * width + col;
        kv[k] = i >= total    ? float4{}
                : t == fresh_at ? reinterpret_cast<const float4 *>(kfresh)[c]
                                : __ldcg(reinterpret_cast<const float4 *>(ksrc + at) + c);
        vv[k] = (i >= total || !vt) ? float4{}
                : t == fresh_at     ? reinterpret_cast<const float4 *>(vfresh)[c]
                                    : __ldcg(reinterpret_cast<const float4 *>(vsrc + at) + c);
    }
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

__global__ void __launch_bounds__(kThreads, 1) k_sparse_attention(Args a) {
    pdl_trigger();
    extern __shared__ __align__(16) float sm[];
    const int units = a.chunks + 1;
    const int kh = blockIdx.x / units, u = blockIdx.x % units;
    const int G = a.H / a.KVH, d = a.d, width = a.KVH * d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kThreads / 32;
    __shared__ int last_unit;
    float *lat = sm;
    float *qs = lat + ((a.latent_dim + 3) & ~3);
    float *knew = qs + G * d, *vnew = knew + d;
    float *kT = vnew + d;                  // [d][kPad]
    float *vt = kT + ((d * kPad + 3) & ~3);  // [kChunk][d]
    float *ps = vt + kChunk * d;           // [G][kChunk]
    float *bscore = ps + G * kChunk;       // block unit: [G][max_blocks]
    int *rank = reinterpret_cast<int *>(bscore + G * a.max_blocks);
    int *kept_s = rank + G * a.max_blocks;  // [G][slots_max]
    float *pen = reinterpret_cast<float *>(kept_s + G * a.slots_max);  // [max_blocks]
    float *ml = pen + a.max_blocks;        // merge: [units][G][2]
    const bool block_unit = u == a.chunks;
    const int newest = a.length - 1;       // window index of the new row
    const int t0 = u * kChunk, n = block_unit ? 0 : max(0, min(kChunk, a.length - t0));

    // 0. before the wait: L2 prefetch of this unit's kv_up rows, window rows, block means
    const int r0 = 2 * d * u / units, r1 = 2 * d * (u + 1) / units;
    const size_t lrow = static_cast<size_t>(a.latent_dim) * (a.kv_dtype == MR_DTYPE_F32 ? 4 : 2);
    if (threadIdx.x == 0) {
        const char *base = static_cast<const char *>(a.kv_up);
        if (r0 < min(r1, d)) prefetch_l2(base + (kh * d + r0) * lrow, (min(r1, d) - r0) * lrow);
        if (max(r0, d) < r1) prefetch_l2(base + (width + kh * d + max(r0, d) - d) * lrow, (r1 - max(r0, d)) * lrow);
        probe(a.probe, kProbeStart);
    }
    if (block_unit) {
        prefetch_rows(a.k_mean + kh * d, width, a.blocks, d);
    } else {
        prefetch_rows(a.k_ring + static_cast<size_t>(a.start + t0) * width + kh * d, width, n, d);
        prefetch_rows(a.v_ring + static_cast<size_t>(a.start + t0) * width + kh * d, width, n, d);
    }
    pdl_wait();
    if (threadIdx.x == 0) probe(a.probe, kProbeWaited);

    // 1. this unit's rows of kv = W_kv_up latent: rows r of head kh's 2d rows
    //    (keys kh*d .., values width + kh*d ..), split evenly over the units
    for (int i = threadIdx.x; i < a.latent_dim; i += kThreads) lat[i] = __ldcg(a.latent + i);
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
                    if (c0 + 32 * k < nv) acc += dot16(w[k], lat + per * (c0 + 32 * k), a.kv_dtype);
            }
        } else {
            for (int j = lane; j < a.latent_dim; j += 32) acc = fmaf(load_weight(rp, a.kv_dtype, j), lat[j], acc);
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
    // 2. the group's queries, normalised and rotated
    for (int g = warp; g < G; g += nwarps) {
        const int h = kh * G + g;
        float *dst = qs + g * d;
        for (int j = lane; j < d; j += 32) dst[j] = __ldcg(a.q + static_cast<size_t>(h) * d + j);
        __syncwarp();
        norm_rope(dst, dst, d, a.split_half, a.position, a.inv_freq);
    }
    const bool needs_new = block_unit || (newest >= t0 && newest < t0 + kChunk);
    bool ok = true;
    if (needs_new) {
        if (threadIdx.x == 0) wait_count(&a.ready[kh], a.seq * units, a.err, a.wait_ns);
        __syncthreads();
        ok = !*reinterpret_cast<volatile int *>(a.err);
        if (ok) {
            for (int j = threadIdx.x; j < d; j += kThreads) {
                knew[j] = __ldcg(a.kv + kh * d + j);
                vnew[j] = __ldcg(a.kv + width + kh * d + j);
            }
            __syncthreads();
            if (warp == 0) norm_rope(knew, knew, d, a.split_half, a.position, a.inv_freq);
        }
    }
    __syncthreads();
    float *part = a.partial + (static_cast<size_t>(kh) * units + u) * G * (d + 2);

    if (ok && !block_unit) {
        // 3a. window keys [t0, t0 + n) of the logical ring (no wrap: the ring spans the context)
        load_tile(kT, vt, a.k_ring, a.v_ring, static_cast<size_t>(a.start + t0), width, kh * d, n, d, newest - t0,
                  knew, vnew);
        __syncthreads();
        for (int i = threadIdx.x; i < G * n; i += kThreads) {
            const int g = i / n, t = i % n;
            ps[g * kChunk + t] = tile_score(qs + g * d, kT, t, d);
        }
        __syncthreads();
        if (threadIdx.x == 0) probe(a.probe, kProbeX5);  // window units: scores done
        // per query head: max, exp and sum (warp g), then the value mix
        for (int g = warp; g < G; g += nwarps) {
            float m = -INFINITY;
            for (int t = lane; t < n; t += 32) m = fmaxf(m, ps[g * kChunk + t]);
            m = warp_max(m);
            float l = 0.f;
            for (int t = lane; t < n; t += 32) {
                const float e = expf(__fsub_rn(ps[g * kChunk + t], m));
                ps[g * kChunk + t] = e;
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
                const float4 p4 = *reinterpret_cast<const float4 *>(ps + g * kChunk + t);
                acc = fmaf(p4.x, vt[t * d + j], acc);
                acc = fmaf(p4.y, vt[(t + 1) * d + j], acc);
                acc = fmaf(p4.z, vt[(t + 2) * d + j], acc);
                acc = fmaf(p4.w, vt[(t + 3) * d + j], acc);
            }
            for (; t < n; ++t) acc = fmaf(ps[g * kChunk + t], vt[t * d + j], acc);
            part[g * (d + 2) + j] = acc;
        }
    } else if (ok) {
        // 3b. block unit: append the new row, the newest block's mean, block scores, top-k
        if (threadIdx.x == 0) probe(a.probe, kProbeX6);  // block unit: past the key / value wait
        const int b = a.blocks - 1;
        const int first = (a.count - 1) % a.block == 0;
        const float inv_n = static_cast<float>(a.count - b * a.block);
        const size_t row = static_cast<size_t>(a.count - 1);
        for (int j = threadIdx.x; j < d; j += kThreads) {
            const size_t at = static_cast<size_t>(kh) * d + j;
            a.k_ring[row * width + at] = knew[j];
            a.v_ring[row * width + at] = vnew[j];
            const float ks = first ? FADD(0.f, knew[j]) : FADD(a.k_bsum[at], knew[j]);
            const float vs = first ? FADD(0.f, vnew[j]) : FADD(a.v_bsum[at], vnew[j]);
            a.k_bsum[at] = ks;
            a.v_bsum[at] = vs;
            knew[j] = __fdiv_rn(ks, inv_n);  // the newest block's mean key / value from here on
            vnew[j] = __fdiv_rn(vs, inv_n);
            a.k_mean[static_cast<size_t>(b) * width + at] = knew[j];
            a.v_mean[static_cast<size_t>(b) * width + at] = vnew[j];
        }
        // the distance penalty of every block column (model.py:220-222), one load round
        for (int bb = threadIdx.x; bb < a.blocks; bb += kThreads)
            pen[bb] = FMUL(a.slope, a.log1p_table[a.position - min((bb + 1) * a.block - 1, a.position)]);
        // block scores minus the penalty; the mean keys through the tile, kChunk blocks at a time
        for (int b0 = 0; b0 < a.blocks; b0 += kChunk) {
            const int nb = min(kChunk, a.blocks - b0);
            __syncthreads();
            load_tile(kT, nullptr, a.k_mean, nullptr, static_cast<size_t>(b0), width, kh * d, nb, d, b - b0, knew,
                      nullptr);
            __syncthreads();
            for (int i = threadIdx.x; i < G * nb; i += kThreads) {
                const int g = i / nb, t = i % nb;
                bscore[g * a.blocks + b0 + t] = __fsub_rn(tile_score(qs + g * d, kT, t, d), pen[b0 + t]);
            }
        }
        __syncthreads();
        // stable descending rank per head (ties to the lower index); the best `slots` stay
        for (int i = threadIdx.x; i < G * a.blocks; i += kThreads) {
            const int g = i / a.blocks, bb = i % a.blocks;
            const float v = bscore[g * a.blocks + bb];
            int r = 0;
            for (int j = 0; j < a.blocks; ++j) {
                const float w = bscore[g * a.blocks + j];
                r += (w > v) || (w == v && j < bb);
            }
            rank[i] = (r < a.slots && v != -INFINITY) ? r : -1;
        }
        __syncthreads();
        // kept ids ascending per head (np.flatnonzero order), -1 padded; their mean values staged
        if (threadIdx.x < G) {
            const int g = threadIdx.x, h = kh * G + g;
            int k = 0;
            for (int bb = 0; bb < a.blocks && k < a.slots_max; ++bb)
                if (rank[g * a.blocks + bb] >= 0) {
                    kept_s[g * a.slots_max + k] = bb;
                    a.kept[h * a.slots_max + k++] = bb;
                }
            for (; k < a.slots_max; ++k) {
                kept_s[g * a.slots_max + k] = -1;
                a.kept[h * a.slots_max + k] = -1;
            }
        }
        __syncthreads();
        float *vk = vt;  // [G][slots_max][d] mean values of the kept blocks
        {
            constexpr int kPer = kChunk * kMaxDim / 4 / kThreads;
            const int total = G * a.slots_max * (d / 4);
            float4 v[kPer];
#pragma unroll
            for (int k = 0; k < kPer; ++k) {
                const int i = threadIdx.x + k * kThreads, gk = i / (d / 4), c = i % (d / 4);
                const int bb = i < total ? kept_s[gk] : -1;
                v[k] = bb < 0    ? float4{}
                       : bb == b ? reinterpret_cast<const float4 *>(vnew)[c]
                                 : __ldcg(reinterpret_cast<const float4 *>(a.v_mean + static_cast<size_t>(bb) * width +
                                                                           kh * d) + c);
            }
#pragma unroll
            for (int k = 0; k < kPer; ++k) {
                const int i = threadIdx.x + k * kThreads;
                if (i < total) reinterpret_cast<float4 *>(vk + (i / (d / 4)) * d)[i % (d / 4)] = v[k];
            }
        }
        __syncthreads();
        for (int g = warp; g < G; g += nwarps) {
            const int *kg = kept_s + g * a.slots_max;
            float m = -INFINITY;
            for (int k = lane; k < a.slots_max; k += 32)
                if (kg[k] >= 0) m = fmaxf(m, bscore[g * a.blocks + kg[k]]);
            m = warp_max(m);
            float l = 0.f;
            for (int k = lane; k < a.slots_max; k += 32)
                if (kg[k] >= 0) l += expf(__fsub_rn(bscore[g * a.blocks + kg[k]], m));
            l = warp_sum(l);
            for (int j = lane; j < d; j += 32) {
                float acc = 0.f;
                if (m != -INFINITY)
                    for (int k = 0; k < a.slots_max; ++k) {
                        if (kg[k] < 0) break;
                        acc = fmaf(expf(__fsub_rn(bscore[g * a.blocks + kg[k]], m)), vk[(g * a.slots_max + k) * d + j],
                                   acc);
                    }
                part[g * (d + 2) + j] = acc;
            }
            if (lane == 0) {
                part[g * (d + 2) + d] = m;
                part[g * (d + 2) + d + 1] = m == -INFINITY ? 0.f : l;
            }
        }
        if (threadIdx.x == 0) probe(a.probe, kProbeX7);  // block unit: done
    }
    // 4. the last unit of this KV head merges every unit's partial softmax
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long before = atomicAdd(&a.done[kh], 1ull);
        last_unit = before == a.seq * units - 1;
        probe(a.probe, kProbeMain);
    }
    __syncthreads();
    if (!last_unit) return;
    __threadfence();
    // every unit's max and sum staged; each thread's weighted values loaded kMergeBatch units at a time
    const float *base = a.partial + static_cast<size_t>(kh) * units * G * (d + 2);
    for (int i = threadIdx.x; i < units * G; i += kThreads) {
        ml[2 * i] = __ldcg(base + i * (d + 2) + d);
        ml[2 * i + 1] = __ldcg(base + i * (d + 2) + d + 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * d; i += kThreads) {
        const int g = i / d, j = i % d;
        float mx = -INFINITY;
        for (int v = 0; v < units; ++v) mx = fmaxf(mx, ml[2 * (v * G + g)]);
        float num = 0.f, den = 0.f;
        for (int v0 = 0; v0 < units; v0 += kMergeBatch) {
            float acc[kMergeBatch];
#pragma unroll
            for (int k = 0; k < kMergeBatch; ++k)
                acc[k] = v0 + k < units ? __ldcg(base + ((v0 + k) * G + g) * (d + 2) + j) : 0.f;
#pragma unroll
            for (int k = 0; k < kMergeBatch; ++k) {
                if (v0 + k >= units) break;
                const float mv = ml[2 * ((v0 + k) * G + g)];
                if (mv == -INFINITY) continue;
                const float f = expf(__fsub_rn(mv, mx));
                num = fmaf(acc[k], f, num);
                den = fmaf(ml[2 * ((v0 + k) * G + g) + 1], f, den);
            }
        }
        a.out[static_cast<size_t>(kh * G + g) * d + j] = __fdiv_rn(num, den);
    }
    __syncthreads();
    if (threadIdx.x == 0) probe(a.probe, kProbeExit);
}

// Shared memory of one unit (floats): latent, q, new k / v, the transposed
// key tile and the value tile (the block unit's mean keys and kept mean
// values), p, the block unit's [G][max_blocks] scores and ranks, [G][slots_max]
// kept ids and [max_blocks] penalties, and the merge's [units][G] max and sum.
inline size_t smem_bytes(int latent_dim, int G, int d, int max_blocks, int slots_max, int units) {
    return (((latent_dim + 3) & ~3) + static_cast<size_t>(G) * d + 2 * d +
            ((static_cast<size_t>(d) * kPad + 3) & ~static_cast<size_t>(3)) + static_cast<size_t>(kChunk) * d +
            static_cast<size_t>(G) * kChunk + 2 * static_cast<size_t>(G) * max_blocks +
            static_cast<size_t>(G) * slots_max + max_blocks + 2 * static_cast<size_t>(units) * G) *
           sizeof(float);
}

}  // namespace attn
