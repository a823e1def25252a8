// Heavy Medium batched prompt (included by heavy.cu only): the token step of
// model.py:192-285 applied to a chunk of T prompt tokens at once, layer by
// layer and inner loop by inner loop, leaving exactly the state the device
// token step continues from (key / value rows, block means, the newest
// block's running sums, the last token's kept blocks and experts).
//
// Per layer and inner loop:
//   RMSNorm(x, a_norm) -> planes -> GEMM q | latent -> planes(latent) -> GEMM kv_up
//   -> per-head q / k norm + RoPE, key / value rows into the rows store
//   -> running block sums of the chunk's positions, block means of the blocks it fills
//   -> sparse attention per token (block scores, top-k, window) -> planes
//   -> GEMM o, x += s o -> RMSNorm(x, f_norm) -> planes -> GEMM router -> routing per token
//   -> tokens sorted by routed expert -> grouped GEMMs gate | up, SwiGLU, down
//   -> dense GEMMs of the shared experts -> rank-order combine, x += s moe.
// GEMMs run on tcgen05 with the activations split into three BF16 parts
// (batch_gemm, prefill.cu), so every product is exact and only the FP32
// accumulation order differs from the token step's; element-wise steps, the
// block sums (in position order), the block scores, the top-k, the routing
// and the combine use the token step's expressions.
#pragma once

namespace hp {

constexpr int kThreads = 256;
constexpr int kRows = 32;     // attention: query rows per CTA (tokens x group heads)
constexpr int kKT = 32;       // attention: keys (or blocks) per tile
constexpr int kMaxSlots = 32;  // kept blocks per query head the attention supports
constexpr int kPT = kRows + 4;  // key-major score / weight rows: four rows' weights in one float4

// x[t] = embedding row of ids[t], widened exactly.
__global__ void k_embed(const int *ids, int T, const void *embed, int dt, int h, float *x) {
    const int t = blockIdx.x;
    const size_t row = static_cast<size_t>(__ldg(ids + t)) * h;
    for (int j = threadIdx.x; j < h; j += blockDim.x) x[static_cast<size_t>(t) * h + j] = load_weight(embed, dt, row + j);
}

// planes[t][j] = split(src[t][j]) for j < cols (no normalisation).
__global__ void k_split(const float *src, int ld, int cols, int T, uint16_t *planes, size_t ps, int lda) {
    const size_t n = static_cast<size_t>(T) * cols;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = i / cols, j = i - t * cols;
        put_planes(planes, ps, t * lda + j, src[t * ld + j]);
    }
}

// One warp per (token, row): rows 0..H-1 the queries (normalised, rotated into
// qh), H..H+KVH-1 the keys (normalised, rotated into the rows store at the
// token's position), H+KVH.. the values (copied there): attn::norm_rope, the
// token step's arithmetic.
__global__ void k_qk(const float *qlat, int ldq, const float *kv, int T, int p0, int H, int KVH, int d, int split_half,
                     const float *inv_freq, float *qh, float *k_rows, float *v_rows) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int per = H + 2 * KVH, width = KVH * d;
    if (warp >= T * per) return;
    const int t = warp / per, r = warp % per, p = p0 + t;
    if (r < H) {
        attn::norm_rope(qlat + static_cast<size_t>(t) * ldq + r * d, qh + (static_cast<size_t>(t) * H + r) * d, d,
                        split_half, p, inv_freq);
    } else if (r < H + KVH) {
        const int kh = r - H;
        attn::norm_rope(kv + static_cast<size_t>(t) * 2 * width + kh * d, k_rows + static_cast<size_t>(p) * width + kh * d,
                        d, split_half, p, inv_freq);
    } else {
        const int kh = r - H - KVH;
        for (int j = lane; j < d; j += 32)
            v_rows[static_cast<size_t>(p) * width + kh * d + j] = kv[static_cast<size_t>(t) * 2 * width + width + kh * d + j];
    }
}

// Running block sums at every position of the chunk, per column, in position
// order (the token step's k_bsum / v_bsum recurrence: a block's first row
// starts from 0, later rows add to the sum; a chunk that starts inside a block
// continues the carried sum).  Each block the chunk reaches gets its mean at
// the chunk's last row in it (the mean the token step would have left), the
// newest block's running sums are carried on.  Thread = (block, column, k|v).
__global__ void k_block_sums(const float *k_rows, const float *v_rows, int T, int p0, int width, int block,
                             float *k_bsum, float *v_bsum, float *k_mean, float *v_mean, float *sum_k, float *sum_v) {
    const int b_first = p0 / block, b_last = (p0 + T - 1) / block;
    const size_t n = static_cast<size_t>(b_last - b_first + 1) * width * 2;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % width), kind = static_cast<int>((i / width) & 1);
        const int b = b_first + static_cast<int>(i / (2 * static_cast<size_t>(width)));
        const float *rows = kind ? v_rows : k_rows;
        float *carry = kind ? v_bsum : k_bsum, *mean = kind ? v_mean : k_mean, *at = kind ? sum_v : sum_k;
        const int lo = max(p0, b * block), hi = min(p0 + T - 1, (b + 1) * block - 1);
        float s = lo % block == 0 ? 0.f : carry[c];
        for (int p = lo; p <= hi; ++p) {
            const float v = rows[static_cast<size_t>(p) * width + c];
            s = p % block == 0 ? FADD(0.f, v) : FADD(s, v);
            at[static_cast<size_t>(p - p0) * width + c] = s;
        }
        mean[static_cast<size_t>(b) * width + c] = __fdiv_rn(s, static_cast<float>(hi - b * block + 1));
        if (b == b_last) carry[c] = s;
    }
}

// The routing of every token (route_block per token, model.py:233-250).
struct RouteRows {
    RouteArgs ra;      // router / chosen / weights / active of token 0; strides below
    int ld_router, T;
};
__global__ void __launch_bounds__(256) k_route(RouteRows a) {
    RouteArgs ra = a.ra;
    const int t = blockIdx.x;
    ra.router += static_cast<size_t>(t) * a.ld_router;
    ra.chosen += static_cast<size_t>(t) * ra.max_k;
    ra.weights += static_cast<size_t>(t) * ra.max_k;
    ra.active += t;
    route_block(ra);
}

// Tokens sorted by routed expert: counts, offsets, each (token, rank) pair's
// row in the sorted order (row_of, -1 past the token's active experts), each
// row's token (token_of), and the tile table of the grouped GEMMs: one entry
// {expert, row0, row_end, 0} per 128 rows of an expert.  One CTA.  The order
// of rows inside an expert is not fixed (atomics); every row is computed on
// its own, so the results are.
__global__ void __launch_bounds__(1024) k_moe_plan(const int *chosen, const int *active, int T, int max_k, int experts,
                                                   int *row_of, int *token_of, int4 *tiles, int *tile_count,
                                                   int max_tiles, int *rows, int *err) {
    __shared__ int count[256], cursor[256];
    for (int e = threadIdx.x; e < experts; e += blockDim.x) count[e] = 0;
    __syncthreads();
    const int n = T * max_k;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int t = i / max_k, k = i % max_k;
        const int e = k < __ldg(active + t) ? __ldg(chosen + i) : -1;
        if (k < __ldg(active + t) && (e < 0 || e >= experts)) atomicCAS(err, 0, 4);
        else if (e >= 0) atomicAdd(&count[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int off = 0, nt = 0;
        for (int e = 0; e < experts; ++e) {
            cursor[e] = off;
            for (int r0 = 0; r0 < count[e] && nt < max_tiles; r0 += kBatchTileRows)
                tiles[nt++] = make_int4(e, off + r0, off + count[e], 0);
            off += count[e];
        }
        *tile_count = nt;
        *rows = off;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int t = i / max_k, k = i % max_k;
        const int e = k < __ldg(active + t) ? __ldg(chosen + i) : -1;
        int row = -1;
        if (e >= 0 && e < experts) {
            row = atomicAdd(&cursor[e], 1);
            token_of[row] = t;
        }
        row_of[i] = row;
    }
}

// dst row r = src row token_of[r] (three planes, 16-byte pieces), r < rows.
__global__ void k_gather(const uint16_t *src, size_t sps, int lds, const int *token_of, const int *rows, int h,
                         uint16_t *dst, size_t dps, int ldd) {
    const int n = __ldg(rows), q = h / 8;
    const size_t total = static_cast<size_t>(n) * q * 3;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int pl = static_cast<int>(i % 3), c = static_cast<int>((i / 3) % q), r = static_cast<int>(i / (3 * q));
        const int t = __ldg(token_of + r);
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src + pl * sps + static_cast<size_t>(t) * lds) + c);
        reinterpret_cast<uint4 *>(dst + pl * dps + static_cast<size_t>(r) * ldd)[c] = v;
    }
}

// planes[r] = split(silu(gate) * up) of gu[r] = gate row | up row, r < *rows
// (or r < T when rows is NULL): the token step's expression.
__global__ void k_swiglu(const float *gu, const int *rows, int T, int f, uint16_t *planes, size_t ps, int ld) {
    const size_t n = static_cast<size_t>(rows ? __ldg(rows) : T) * f;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = i / f, j = i - r * f;
        const float g = gu[r * 2 * f + j], u = gu[r * 2 * f + f + j];
        put_planes(planes, ps, r * ld + j, FMUL(__fdiv_rn(g, FADD(1.0f, expf(-g))), u));
    }
}

// x[t] += scale * (sum over the token's experts in rank order of weight *
// down row, then each shared expert's down row * shared_scale): the token
// step's combine (model.py:251-255).
__global__ void k_combine(float *x, int T, int h, const int *active, const float *weights, const int *row_of, int max_k,
                          const float *routed, const float *shared_out, int shared, float shared_scale, float scale) {
    const size_t n = static_cast<size_t>(T) * h;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i / h), c = static_cast<int>(i % h);
        const int act = __ldg(active + t);
        float res = 0.f;
        for (int k = 0; k < act; ++k) {
            const int r = __ldg(row_of + t * max_k + k);
            if (r < 0) continue;  // an id outside the expert table (reported through err by k_moe_plan)
            res = FADD(res, FMUL(__ldg(weights + t * max_k + k), routed[static_cast<size_t>(r) * h + c]));
        }
        for (int j = 0; j < shared; ++j)
            res = FADD(res, FMUL(shared_scale, shared_out[(static_cast<size_t>(j) * T + t) * h + c]));
        x[i] = FADD(x[i], FMUL(scale, res));
    }
}


// ---- sparse attention of a chunk ------------------------------------------------------------
struct AttnArgs {
    const float *qh;               // [T][H * d] normalised, rotated queries
    const float *k_rows, *v_rows;  // [context][width] every position's key / value
    const float *k_mean, *v_mean;  // [blocks][width] block means (final for every block before a token's own)
    const float *sum_k, *sum_v;    // [T][width] running sums of each token's own block at the token
    const float *log1p_table;
    float slope;
    int T, p0, H, KVH, d, window, block, slots, slots_max, nb;  // nb: blocks of the chunk's last token
    uint16_t *planes;              // output: planes of the o projection's input [3][T][ld]
    size_t ps;
    int ld;
    int *kept_last;                // [H][slots_max]: the chunk's last token's kept blocks
    float *block_state;            // or NULL: stop after the block part and leave each row's softmax
                                   // state here ([T * H][d + 2]: weighted values, max, sum) for k_window_tc
};

// q . k / sqrt(d) with the token step's association (attn::tile_score): four
// FMA chains over the columns in order, (a0 + a1) + (a2 + a3).
__device__ __forceinline__ float score4(const float *q, const float *k, int d, float sqrt_d) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int j = 0; j < d; j += 4) {
        const float4 q4 = *reinterpret_cast<const float4 *>(q + j), k4 = *reinterpret_cast<const float4 *>(k + j);
        a0 = fmaf(q4.x, k4.x, a0);
        a1 = fmaf(q4.y, k4.y, a1);
        a2 = fmaf(q4.z, k4.z, a2);
        a3 = fmaf(q4.w, k4.w, a3);
    }
    return __fdiv_rn((a0 + a1) + (a2 + a3), sqrt_d);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}

// CTA = (QT consecutive tokens, KV head kh); rows r = (token, group head).
// A. Block part (model.py:210-226 per token): every block's mean key scored
//    against the row's query minus the distance penalty (the token's own,
//    unfinished block from its running sum), the best `slots` kept (larger
//    score first, ties to the lower block, as the stable argsort), and their
//    softmax terms over the blocks' mean values, in ascending block order,
//    become the row's starting online-softmax state.
// B. Window part: keys (p - window, p] in tiles of 32 (double-buffered
//    cp.async), online softmax continued.  Output rows as BF16x3 planes.
__global__ void __launch_bounds__(kThreads) k_attention(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    const int G = a.H / a.KVH, QT = kRows / G, kh = blockIdx.y, t0 = blockIdx.x * QT;
    const int nt = min(QT, a.T - t0), R = nt * G, d = a.d, width = a.KVH * d, ks = d + 4, dq = d / 4;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float *q = sm;                        // [kRows][d + 4]
    float *kt = q + kRows * ks;           // [2][kKT][d + 4]
    float *vt = kt + 2 * kKT * ks;        // [2][kKT][d]; phase A: each token's own block mean key | value
    float *st = vt + 2 * kKT * d;         // [kKT][kPT] scores, then weights, key-major
    float *mrow = st + kKT * kPT, *lrow = mrow + kRows, *corr = lrow + kRows;  // corr: 16-byte aligned
    float *bscore = corr + kRows;         // [kRows][nb]
    float *ksc = bscore + static_cast<size_t>(kRows) * a.nb;  // [kRows][kMaxSlots] kept scores
    int *kid = reinterpret_cast<int *>(ksc + kRows * kMaxSlots);  // [kRows][kMaxSlots] kept blocks, ascending
    int *nkept = kid + kRows * kMaxSlots;                       // [kRows]
    float *cur_k = vt, *cur_v = vt + QT * d;
    const int p_first = a.p0 + t0, p_last = p_first + nt - 1;
    const int nb = p_last / a.block + 1;  // blocks of the CTA's last token
    const float sqrt_d = __fsqrt_rn(static_cast<float>(d));

    for (int e = tid; e < kRows * d; e += kThreads) {
        const int r = e / d, j = e - r * d, tt = r / G, g = r - tt * G;
        q[r * ks + j] = r < R ? __ldg(a.qh + (static_cast<size_t>(t0 + tt) * a.H + kh * G + g) * d + j) : 0.f;
    }
    for (int e = tid; e < nt * d; e += kThreads) {  // each token's own block: its running mean at the token
        const int tt = e / d, j = e - tt * d, p = p_first + tt;
        const float n = static_cast<float>(p - (p / a.block) * a.block + 1);
        const size_t at = static_cast<size_t>(t0 + tt) * width + kh * d + j;
        cur_k[tt * d + j] = __fdiv_rn(__ldg(a.sum_k + at), n);
        cur_v[tt * d + j] = __fdiv_rn(__ldg(a.sum_v + at), n);
    }
    const int sr = tid >> 3, sk = tid & 7;  // score mapping: row sr, keys sk, sk + 8, sk + 16, sk + 24
    // A1. block scores, kKT block means at a time (the token's own block is scored below)
    for (int b0 = 0; b0 < nb; b0 += kKT) {
        const int nbt = min(kKT, nb - b0);
        __syncthreads();
        for (int e = tid; e < nbt * dq; e += kThreads) {
            const int kk = e / dq, j = (e - kk * dq) * 4;
            *reinterpret_cast<float4 *>(kt + kk * ks + j) =
                __ldg(reinterpret_cast<const float4 *>(a.k_mean + static_cast<size_t>(b0 + kk) * width + kh * d + j));
        }
        __syncthreads();
        if (sr < R) {
            const int p = p_first + sr / G, own = p / a.block;
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int kk = sk + 8 * y, b = b0 + kk;
                if (kk >= nbt) continue;
                float v = -INFINITY;
                if (b < own) {
                    v = __fsub_rn(score4(q + sr * ks, kt + kk * ks, d, sqrt_d),
                                  FMUL(a.slope, __ldg(a.log1p_table + p - min((b + 1) * a.block - 1, p))));
                }
                bscore[static_cast<size_t>(sr) * a.nb + b] = v;
            }
        }
    }
    __syncthreads();
    for (int r = tid; r < R; r += kThreads) {  // A2. the token's own block
        const int tt = r / G, p = p_first + tt, own = p / a.block;
        bscore[static_cast<size_t>(r) * a.nb + own] =
            __fsub_rn(score4(q + r * ks, cur_k + tt * d, d, sqrt_d), FMUL(a.slope, __ldg(a.log1p_table + 0)));
    }
    __syncthreads();
    // A3. the best `slots` blocks of each row: repeated warp argmax (larger score, then lower block)
    for (int x = 0; x < kRows / 8; ++x) {
        const int r = warp + 8 * x;
        if (r >= R) continue;
        const int p = p_first + r / G, nbr = p / a.block + 1, want = min(a.slots, nbr);
        float *row = bscore + static_cast<size_t>(r) * a.nb;
        int n = 0;
        for (; n < want; ++n) {
            float best = -INFINITY;
            int bi = 0x7fffffff;
            for (int b = lane; b < nbr; b += 32) {
                const float v = row[b];
                if (v != -INFINITY && (v > best || (v == best && b < bi))) {
                    best = v;
                    bi = b;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ob > best || (ob == best && oi < bi)) {
                    best = ob;
                    bi = oi;
                }
            }
            if (bi == 0x7fffffff) break;
            if (lane == 0) {
                kid[r * kMaxSlots + n] = bi;
                ksc[r * kMaxSlots + n] = best;
            }
            if (lane == (bi & 31)) row[bi] = -INFINITY;
            __syncwarp();
        }
        if (lane == 0) {  // ascending block order (np.flatnonzero), as the token step keeps them
            for (int i = 1; i < n; ++i)
                for (int j = i; j > 0 && kid[r * kMaxSlots + j - 1] > kid[r * kMaxSlots + j]; --j) {
                    const int ti = kid[r * kMaxSlots + j];
                    const float ts = ksc[r * kMaxSlots + j];
                    kid[r * kMaxSlots + j] = kid[r * kMaxSlots + j - 1];
                    ksc[r * kMaxSlots + j] = ksc[r * kMaxSlots + j - 1];
                    kid[r * kMaxSlots + j - 1] = ti;
                    ksc[r * kMaxSlots + j - 1] = ts;
                }
            nkept[r] = n;
            if (t0 + r / G == a.T - 1) {
                const int h = kh * G + r % G;
                for (int i = 0; i < a.slots_max; ++i) a.kept_last[h * a.slots_max + i] = i < n ? kid[r * kMaxSlots + i] : -1;
            }
        }
    }
    __syncthreads();
    // A4. the kept blocks' softmax terms: the rows' starting state
    for (int r = tid; r < kRows; r += kThreads) {
        float m = -INFINITY, l = 0.f;
        if (r < R) {
            for (int i = 0; i < nkept[r]; ++i) m = fmaxf(m, ksc[r * kMaxSlots + i]);
            for (int i = 0; i < nkept[r]; ++i) l += expf(__fsub_rn(ksc[r * kMaxSlots + i], m));
        }
        mrow[r] = m;
        lrow[r] = l;
    }
    __syncthreads();
    // the output: thread = (four rows 4 rq .., four dims 4 dq4 ..), accumulators in registers
    const int rq = tid >> 5, dq4 = tid & 31;
    const bool has_dims = 4 * dq4 < d;
    float acc[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x) {
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
        const int r = 4 * rq + x;
        if (r >= R || !has_dims) continue;
        const int tt = r / G, own = (p_first + tt) / a.block;
        for (int i = 0; i < nkept[r]; ++i) {
            const int bb = kid[r * kMaxSlots + i];
            const float w = expf(__fsub_rn(ksc[r * kMaxSlots + i], mrow[r]));
            const float *vs = bb == own ? cur_v + tt * d : a.v_mean + static_cast<size_t>(bb) * width + kh * d;
#pragma unroll
            for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(w, vs[4 * dq4 + y], acc[x][y]);
        }
    }
    if (a.block_state) {  // the window runs on the tensor cores (k_window_tc), from this state
        if (!has_dims) return;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const int r = 4 * rq + x;
            if (r >= R) continue;
            const int tt = r / G, g = r - tt * G;
            float *row = a.block_state + (static_cast<size_t>(t0 + tt) * a.H + kh * G + g) * (d + 2);
#pragma unroll
            for (int y = 0; y < 4; ++y) row[4 * dq4 + y] = acc[x][y];
            if (dq4 == 0) {
                row[d] = mrow[r];
                row[d + 1] = lrow[r];
            }
        }
        return;
    }
    __syncthreads();  // phase A's means in vt are read; the window tiles take it over
    // B. the window (p - window, p] of every row
    const int lo = max(0, p_first - a.window + 1);
    auto issue = [&](int kb, int buf) {
        const int nk = min(kKT, p_last + 1 - kb);
        for (int e = tid; e < nk * dq; e += kThreads) {
            const int kk = e / dq, j = (e - kk * dq) * 4;
            const size_t row = static_cast<size_t>(kb + kk) * width + kh * d + j;
            cp_async16(kt + (buf * kKT + kk) * ks + j, a.k_rows + row);
            cp_async16(vt + (buf * kKT + kk) * d + j, a.v_rows + row);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(lo, 0);
    int buf = 0;
    for (int kb = lo; kb <= p_last; kb += kKT, buf ^= 1) {
        const int nk = min(kKT, p_last + 1 - kb);
        if (kb + kKT <= p_last) {
            issue(kb + kKT, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float *ktb = kt + buf * kKT * ks, *vtb = vt + buf * kKT * d;
        {  // scores of row sr against keys sk, sk + 8, sk + 16, sk + 24: one query load per four keys,
           // each score in the token step's association (four chains, (a0 + a1) + (a2 + a3))
            float c[4][4];
#pragma unroll
            for (int y = 0; y < 4; ++y)
#pragma unroll
                for (int z = 0; z < 4; ++z) c[y][z] = 0.f;
            for (int j = 0; j < d; j += 4) {
                const float4 q4 = *reinterpret_cast<const float4 *>(q + sr * ks + j);
#pragma unroll
                for (int y = 0; y < 4; ++y) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(ktb + (sk + 8 * y) * ks + j);
                    c[y][0] = fmaf(q4.x, k4.x, c[y][0]);
                    c[y][1] = fmaf(q4.y, k4.y, c[y][1]);
                    c[y][2] = fmaf(q4.z, k4.z, c[y][2]);
                    c[y][3] = fmaf(q4.w, k4.w, c[y][3]);
                }
            }
            const int p = p_first + sr / G;
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int kk = sk + 8 * y, pos = kb + kk;
                const bool live = sr < R && kk < nk && pos <= p && pos > p - a.window;
                st[kk * kPT + sr] = live ? __fdiv_rn((c[y][0] + c[y][1]) + (c[y][2] + c[y][3]), sqrt_d) : -INFINITY;
            }
        }
        __syncthreads();
        {  // online softmax: warp w updates rows w, w + 8, w + 16, w + 24, one key per lane
            float v[4], mt[4], pr[4], sum[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                v[x] = st[lane * kPT + warp + 8 * x];
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
                pr[x] = v[x] == -INFINITY ? 0.f : expf(__fsub_rn(v[x], m_new));
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
                st[lane * kPT + r] = pr[x];
                if (lane == 0) {
                    const float m_old = mrow[r];
                    const float cf = m_old == -INFINITY ? 0.f : expf(__fsub_rn(m_old, mt[x]));
                    corr[r] = cf;
                    lrow[r] = fmaf(lrow[r], cf, sum[x]);
                    mrow[r] = mt[x];
                }
            }
        }
        __syncthreads();
        if (has_dims && 4 * rq < R) {  // value mix: the four rows' weights of a key in one broadcast load
            const float4 cr = *reinterpret_cast<const float4 *>(corr + 4 * rq);
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                acc[0][y] *= cr.x;
                acc[1][y] *= cr.y;
                acc[2][y] *= cr.z;
                acc[3][y] *= cr.w;
            }
            for (int kk = 0; kk < nk; ++kk) {
                const float4 w4 = *reinterpret_cast<const float4 *>(st + kk * kPT + 4 * rq);
                const float4 vv = *reinterpret_cast<const float4 *>(vtb + kk * d + 4 * dq4);
                const float wx[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    acc[x][0] = fmaf(wx[x], vv.x, acc[x][0]);
                    acc[x][1] = fmaf(wx[x], vv.y, acc[x][1]);
                    acc[x][2] = fmaf(wx[x], vv.z, acc[x][2]);
                    acc[x][3] = fmaf(wx[x], vv.w, acc[x][3]);
                }
            }
        }
        __syncthreads();  // every reader of buffer buf is done before it is refilled
    }
    if (!has_dims) return;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
        const int r = 4 * rq + x;
        if (r >= R) continue;
        const int tt = r / G, g = r - tt * G;
#pragma unroll
        for (int y = 0; y < 4; ++y)
            put_planes(a.planes, a.ps, static_cast<size_t>(t0 + tt) * a.ld + (kh * G + g) * d + 4 * dq4 + y,
                       __fdiv_rn(acc[x][y], lrow[r]));
    }
}

// ---- the window part on the tensor cores ------------------------------------------------
// CTA = 128 rows (128 / G tokens x the G query heads of KV head kh), two threads
// per row (its TMEM lane, from warps w and w + 4: half the output dims each).  Per tile of 64 keys of the rows' windows:
//   S = Q K^T   (M 128, N 64, K 128): Q and K as three BF16 parts each, the six
//               products down to 2^-16 x 2^-8 (Qh Kh, Qh Km, Qm Kh, Qh Kl, Ql Kh, Qm Km)
//   softmax     each thread its row: scale, window mask, running max / sum (online)
//   O_t = P V   (M 128, N 128, K 64): P (into the key tile's space) and V^T, three parts each
//   o = o * correction + O_t in registers.
// Operands are written by the threads straight into the 128-byte-swizzled K-major
// layout (tc::sw128_offset) and read by tcgen05.mma from shared memory; S and O_t
// accumulate in TMEM.  The state starts from the block part's (k_attention with
// block_state), so the result is the softmax over kept blocks and window together.
struct WindowArgs {
    const float *qh;               // [T][H * d] normalised, rotated queries
    const uint8_t *kv_planes;      // k_kv_planes: per 64-key block from block0 and KV head, K then V^T tiles
    int block0;                    // the first 64-key block held there
    const float *block_state;      // [T * H][d + 2]
    int T, p0, H, KVH, d, window;
    uint16_t *planes;              // output: planes of the o projection's input [3][T][ld]
    size_t ps;
    int ld;
    int *err;                      // a bounded wait gave up
};
constexpr int kWRows = 128, kWKeys = 64, kWThreads = 256, kWDim = 128;
constexpr uint32_t kQPlane = 2 * 16384;  // 128 rows x 128 dims: two 64-wide atoms
constexpr uint32_t kKPlane = 2 * 8192;   // 64 keys x 128 dims (the same space: P, 128 rows x 64 keys)
constexpr uint32_t kVPlane = 16384;      // V^T: 128 dims x 64 keys
constexpr size_t kWindowSmem = 1024 + 3 * kQPlane + 3 * kKPlane + 3 * kVPlane + 64;

// Three BF16 parts of eight values (x = p0 + p1 + p2 exactly), each as 16 bytes.
__device__ __forceinline__ void split8(const float (&v)[8], uint4 (&part)[3]) {
    uint32_t w[3][4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        uint16_t h[2][3];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float x = v[i + e];
            const uint16_t a0 = bf16_bits(x);
            const float r1 = __fsub_rn(x, bf16_value(a0));
            const uint16_t a1 = bf16_bits(r1);
            const uint16_t a2 = bf16_bits(__fsub_rn(r1, bf16_value(a1)));
            h[e][0] = a0;
            h[e][1] = a1;
            h[e][2] = a2;
        }
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) w[pl][i / 2] = static_cast<uint32_t>(h[0][pl]) | (static_cast<uint32_t>(h[1][pl]) << 16);
    }
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) part[pl] = make_uint4(w[pl][0], w[pl][1], w[pl][2], w[pl][3]);
}

// Key and value tiles in the window kernel's shared-memory layout, built once per
// layer and loop for every 64-key block a chunk's windows reach: per (block,
// KV head) the three parts of K (64 keys x 128 dims, two 64-dim atoms) and of
// V^T (128 dims x 64 keys), 96 KB, copied by the window kernel as they are.
// Keys past `keys` (the chunk's end) are zero.
constexpr size_t kTileBytes = 3 * kKPlane + 3 * kVPlane;
__host__ __device__ __forceinline__ size_t kv_tile_offset(int block, int KVH, int kh) {
    return (static_cast<size_t>(block) * KVH + kh) * kTileBytes;
}
__global__ void __launch_bounds__(256) k_kv_planes(const float *k_rows, const float *v_rows, int KVH, int block0,
                                                   int keys, uint8_t *planes) {
    const int blk = block0 + static_cast<int>(blockIdx.x) / KVH, kh = blockIdx.x % KVH, tid = threadIdx.x;
    const int width = KVH * kWDim, kb = blk * kWKeys;
    uint8_t *tile = planes + kv_tile_offset(blockIdx.x / KVH, KVH, kh);
    {  // K: thread = (key, 32 dims)
        const int kk = tid >> 2, q4 = tid & 3, atom = q4 >> 1;
        const bool live = kb + kk < keys;
        const float *src = k_rows + static_cast<size_t>(kb + kk) * width + kh * kWDim + q4 * 32;
        float4 x[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) x[c] = live ? __ldcg(reinterpret_cast<const float4 *>(src) + c) : float4{};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float v[8] = {x[2 * c].x, x[2 * c].y, x[2 * c].z, x[2 * c].w,
                                x[2 * c + 1].x, x[2 * c + 1].y, x[2 * c + 1].z, x[2 * c + 1].w};
            uint4 part[3];
            split8(v, part);
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
                *reinterpret_cast<uint4 *>(tile + pl * kKPlane + atom * 8192 +
                                           tc::sw128_offset(kk, (q4 & 1) * 32 + c * 8)) = part[pl];
        }
    }
    {  // V^T: thread = (dim j, 32 keys)
        const int j = tid & 127, k0 = (tid >> 7) * 32;
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
            x[i] = kb + k0 + i < keys ? __ldcg(v_rows + static_cast<size_t>(kb + k0 + i) * width + kh * kWDim + j) : 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float v[8] = {x[8 * c], x[8 * c + 1], x[8 * c + 2], x[8 * c + 3],
                                x[8 * c + 4], x[8 * c + 5], x[8 * c + 6], x[8 * c + 7]};
            uint4 part[3];
            split8(v, part);
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
                *reinterpret_cast<uint4 *>(tile + 3 * kKPlane + pl * kVPlane + tc::sw128_offset(j, k0 + c * 8)) = part[pl];
        }
    }
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::saddr(dst)),
                 "l"(src), "r"(bytes), "r"(tc::saddr(bar))
                 : "memory");
}

__global__ void __launch_bounds__(kWThreads, 1) k_window_tc(WindowArgs a) {
    extern __shared__ uint8_t w_raw[];
    uint8_t *qs = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(w_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *kp = qs + 3 * kQPlane;  // the key tile, then (after S) the weights P
    uint8_t *vt = kp + 3 * kKPlane;
    // [0] S done, [1] O done, [2] the key tile landed, [3] the value tile landed
    uint64_t *bar = reinterpret_cast<uint64_t *>(vt + 3 * kVPlane);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 4);
    const int G = a.H / a.KVH, QT = kWRows / G, kh = blockIdx.y, t0 = blockIdx.x * QT;
    const int nt = min(QT, a.T - t0), R = nt * G;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // two threads per row (TMEM lane): warps w and w + 4; `half` picks the output dims and P chunks
    const int r = (warp & 3) * 32 + lane, half = warp >> 2, tt = r / G, g = r - tt * G;
    const bool live = r < R;
    const int p = a.p0 + t0 + tt, p_first = a.p0 + t0, p_last = p_first + nt - 1;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc::saddr(&bar[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc::saddr(&bar[1])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc::saddr(&bar[2])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc::saddr(&bar[3])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // S: columns 0..63, O_t: 128..255
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(tc::saddr(tslot)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the row's query (this thread: the 64-dim atom `half`) as three parts, all loads first
    // (times 1/sqrt(d): the scores come out of the tensor cores scaled)
    const size_t qrow = (static_cast<size_t>(t0 + tt) * a.H + kh * G + g) * kWDim;
    {
        const float inv_sqrt_d = __frcp_rn(__fsqrt_rn(static_cast<float>(kWDim)));
        float4 x[16];
#pragma unroll
        for (int c = 0; c < 16; ++c)
            x[c] = live ? __ldg(reinterpret_cast<const float4 *>(a.qh + qrow + half * 64) + c) : float4{};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float v[8] = {x[2 * c].x, x[2 * c].y, x[2 * c].z, x[2 * c].w,
                          x[2 * c + 1].x, x[2 * c + 1].y, x[2 * c + 1].z, x[2 * c + 1].w};
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = FMUL(v[i], inv_sqrt_d);
            uint4 part[3];
            split8(v, part);
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
                *reinterpret_cast<uint4 *>(qs + pl * kQPlane + half * 16384 + tc::sw128_offset(r, c * 8)) = part[pl];
        }
    }
    // the block part's state: weighted values (this thread's 64 dims), max, sum
    constexpr int kHalf = kWDim / 2;
    float o[kHalf];
    float m = -INFINITY, l = 0.f;
    {
        const float *bs = a.block_state + (static_cast<size_t>(t0 + tt) * a.H + kh * G + g) * (kWDim + 2);
#pragma unroll
        for (int j = 0; j < kHalf; ++j) o[j] = live ? bs[half * kHalf + j] : 0.f;
        if (live) {
            m = bs[kWDim];
            l = bs[kWDim + 1];
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tslot, lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int lo = max(0, p_first - a.window + 1);
    bool ok = true;
    int tile = 0;
    for (int kb = (lo / kWKeys) * kWKeys; kb <= p_last && ok; kb += kWKeys, ++tile) {
        const int nk = min(kWKeys, p_last + 1 - kb);
        // this block's key / value tiles, as built by k_kv_planes (after every reader of the last tile's
        // P and V^T is done: the barrier at the end of the previous iteration)
        // (keys and values on their own barriers: the S products start while V^T still lands)
        if (tid == 0) {
            const uint8_t *src = a.kv_planes + kv_tile_offset(kb / kWKeys - a.block0, a.KVH, kh);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::saddr(&bar[2])),
                         "r"(static_cast<uint32_t>(3 * kKPlane))
                         : "memory");
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::saddr(&bar[3])),
                         "r"(static_cast<uint32_t>(3 * kVPlane))
                         : "memory");
            bulk_load(kp, src, 3 * kKPlane, &bar[2]);
            bulk_load(vt, src + 3 * kKPlane, 3 * kVPlane, &bar[3]);
        }
        ok = __syncthreads_and(tc::wait(&bar[2], tile & 1, a.err));
        if (!ok) break;
        // the operands are visible to the tensor cores' (async) proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0) {
            const int combos[6][2] = {{0, 0}, {0, 1}, {1, 0}, {0, 2}, {2, 0}, {1, 1}};
            const uint32_t qb = tc::saddr(qs), kbase = tc::saddr(kp);
            bool first = true;
#pragma unroll
            for (int cmb = 0; cmb < 6; ++cmb)
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint64_t ad = tc::sw128_desc(qb + combos[cmb][0] * kQPlane + (ks >> 2) * 16384 + (ks & 3) * 32);
                    const uint64_t bd = tc::sw128_desc(kbase + combos[cmb][1] * kKPlane + (ks >> 2) * 8192 + (ks & 3) * 32);
                    tc::mma(tmem, ad, bd, tc::idesc(128, 64), !first);
                    first = false;
                }
            tc::commit(&bar[0]);
        }
        ok = __syncthreads_and(tc::wait(&bar[0], tile & 1, a.err));
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // softmax of this row over the tile (both threads of a row compute the same values)
        float sc[kWKeys];
        {
            uint32_t u[32];
            tc::tmem_ld32(lane_base, u);
#pragma unroll
            for (int k = 0; k < 32; ++k) sc[k] = __uint_as_float(u[k]);
            tc::tmem_ld32(lane_base + 32, u);
#pragma unroll
            for (int k = 0; k < 32; ++k) sc[32 + k] = __uint_as_float(u[k]);
        }
        float mt = m;
#pragma unroll
        for (int k = 0; k < kWKeys; ++k) {
            const int pos = kb + k;
            const bool valid = live && k < nk && pos <= p && pos > p - a.window;
            if (!valid) sc[k] = -INFINITY;
            mt = fmaxf(mt, sc[k]);
        }
        const float corr = m == -INFINITY ? 0.f : expf(__fsub_rn(m, mt));
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < kWKeys; ++k) {
            sc[k] = sc[k] == -INFINITY ? 0.f : expf(__fsub_rn(sc[k], mt));
            sum += sc[k];
        }
        l = fmaf(l, corr, sum);
        m = mt;
        // P into the key tile's space, three parts: this thread its half of the row's chunks
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int cc = half * 4 + c;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = sc[cc * 8 + i];
            uint4 part[3];
            split8(v, part);
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
                *reinterpret_cast<uint4 *>(kp + pl * kKPlane + tc::sw128_offset(r, cc * 8)) = part[pl];
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        bool v_ok = true;
        if (tid == 0 && (v_ok = tc::wait(&bar[3], tile & 1, a.err))) {  // the value tile, then P V^T
            const int combos[6][2] = {{0, 0}, {0, 1}, {1, 0}, {0, 2}, {2, 0}, {1, 1}};
            const uint32_t pb = tc::saddr(kp), vb = tc::saddr(vt);
            bool first = true;
#pragma unroll
            for (int cmb = 0; cmb < 6; ++cmb)
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t ad = tc::sw128_desc(pb + combos[cmb][0] * kKPlane + ks * 32);
                    const uint64_t bd = tc::sw128_desc(vb + combos[cmb][1] * kVPlane + ks * 32);
                    tc::mma(tmem + 128, ad, bd, tc::idesc(128, 128), !first);
                    first = false;
                }
            tc::commit(&bar[1]);
        }
        ok = __syncthreads_and(v_ok);
        if (!ok) break;
        ok = __syncthreads_and(tc::wait(&bar[1], tile & 1, a.err));
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int c = 0; c < kHalf; c += 32) {
            uint32_t u[32];
            tc::tmem_ld32(lane_base + 128 + half * kHalf + c, u);
#pragma unroll
            for (int k = 0; k < 32; ++k) o[c + k] = fmaf(o[c + k], corr, __uint_as_float(u[k]));
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();  // every thread has its O_t and is done with P: the next tile may overwrite them
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    if (ok && live) {
#pragma unroll
        for (int j = 0; j < kHalf; ++j)
            put_planes(a.planes, a.ps,
                       static_cast<size_t>(t0 + tt) * a.ld + (kh * G + g) * kWDim + half * kHalf + j,
                       __fdiv_rn(o[j], l));
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

// Shared memory of k_attention for head dim d and nb blocks.
inline size_t attention_smem(int d, int nb) {
    return sizeof(float) * (static_cast<size_t>(kRows) * (d + 4) + 2 * kKT * (d + 4) + 2 * static_cast<size_t>(kKT) * d +
                            kKT * kPT + 3 * kRows + static_cast<size_t>(kRows) * nb + 2 * kRows * kMaxSlots + kRows);
}

}  // namespace hp
