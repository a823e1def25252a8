// Work between two decode steps for the two families whose attention caches
// change shape beyond a ring (included by engine.cu only):
//
// * flashnano-1.6 chunk relays (model.py:118-144): every cbr_chunk_size
//   tokens each layer pools the chunk's normalised inputs into cbr_slots relay
//   rows (scores against the normalised relay queries, softmax over the
//   chunk, probability-weighted rows and rounded anchor positions), projects
//   them to keys (k_norm, RoPE at the anchors) and values, and appends them
//   to the layer's relay rows, which the decode kernel's attention reads
//   after the ring (AttnPhase::relay_*).  The decode kernel's q | k | v phase
//   leaves each token's raw layer input in `pending` (GemvPhase::save_in).
//
// * FlashLighting with memory slots (model.py:170-186): a latent row that
//   leaves the attention window joins the layer's memory rows; when memory
//   would exceed memory_slots, its two oldest rows merge, weighted by how
//   many tokens each stands for, at the weighted mean position (rounded).
//   Memory rows are the decode kernel's relay rows: their keys (normalised,
//   rotated at the row's position) and values.  Only a merged row's key and
//   value are new; an absorbed row's are the ring's.  The decode kernel's
//   k | v phase leaves each token's raw latent in `lat_ring`; the row that
//   will leave the window at the next token is copied aside (the stash)
//   before that token's step overwrites its ring slot.
//
// Launched after every decode step, on the step's stream: k_aux_plan (one
// thread per layer: which work is due at the position just processed, the
// float32 bookkeeping of positions and counts), then the kernels that move
// the data (FlashLighting: k_aux_merge, k_aux_move, k_aux_merged_kv;
// flashnano-1.6: k_cbr_scores, k_cbr_pool, k_cbr_kv).  A step that did not
// run (stopped, error) leaves the position unchanged, and the plan does
// nothing twice for one position.
#pragma once

namespace mr {
namespace aux {

// float32 arithmetic with one rounding per operation (no contraction), as the reference kernels
__device__ __forceinline__ float FADD(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float FMUL(float a, float b) { return __fmul_rn(a, b); }

constexpr int kThreads = 256;

struct Layer {
    // flashnano-1.6
    float *pending;          // [chunk][hidden] raw layer inputs
    const void *a_norm;      // input norm gain (the layer's a_norm)
    int a_norm_dt;
    const float *queries;    // [slots][hidden] normalised relay queries
    float *u;                // [chunk][hidden] normalised inputs (scratch)
    float *scores;           // [slots][chunk]
    float *pooled;           // [slots][hidden]
    float *anchors;          // [slots]
    int relay_base;          // first relay row written by the pooling now due
    // both
    const void *wk, *wv;     // [kv_width][in] key / value projections (in: hidden or latent)
    int w_dt;
    int kv_heads, kv_width;  // this layer's
    const void *k_norm;      // per-head key norm gain
    int k_norm_dt;
    float *relay_k, *relay_v;  // [kv_heads][relay_cap][d]
    int *relay_count;        // rows the decode kernel attends after the ring
    int relay_cap;
    int due;                 // set by k_aux_plan: 1 pooling (nano-1.6) / bit 0 absorb, bit 1 merge, bit 2 stash
    int last_pos;            // last position planned
    // FlashLighting memory
    float *lat_ring;         // [window][latent] raw latents
    const void *latent_norm;
    int latent_norm_dt;
    const float *k_cache, *v_cache;  // [kv_heads][window][d] the ring of keys / values
    float *mem_lat;          // [memory_slots][latent] memory latents (normalised, or merged)
    int *mem_pos;            // [memory_slots] positions, logical order
    float *mem_cnt;          // [memory_slots] tokens each stands for, logical order
    int *mem_slot;           // [memory_slots] physical row of each logical row
    float *stash_k, *stash_v, *stash_lat;  // [2][kv_width], [2][latent]: rows leaving the window
    int stash_pos[2];        // their positions (-1: none)
    // this step's plan (k_aux_plan -> k_aux_move / k_aux_project)
    int src0, src1;          // merge inputs: physical memory rows (-1: the stash of parity `stash_in`)
    float wa, wb;            // their counts
    int dst;                 // physical row receiving the merged latent (its key / value recomputed)
    int absorb_to;           // physical row receiving the stash as it is (-1: none)
    int stash_in, stash_out; // stash parities: the one absorbed now, the one filled now
    int merged_pos;
};

struct Model {
    int layers, hidden, d, split_half;
    float norm_eps;
    const float *inv_freq;
    // flashnano-1.6
    int chunk, slots;
    // FlashLighting memory
    int window, memory_slots, latent;
    int lighting;            // 1: FlashLighting memory slots, 0: flashnano-1.6 relays
};

// float32 RMSNorm factor of n values as kernels.cl:19-28 (sum of squares in
// order, one thread), and the normalised value (x * scale) * gain.
__device__ __forceinline__ float rms_scale(const float *x, int n, float eps) {
    float ss = 0.f;
    for (int j = 0; j < n; ++j) ss = FADD(ss, FMUL(x[j], x[j]));
    return __fdiv_rn(1.0f, __fsqrt_rn(FADD(__fdiv_rn(ss, static_cast<float>(n)), eps)));
}

// ---- the plan: one thread per layer ----------------------------------------------------
__global__ void k_aux_plan(Model m, Layer *layers, const StepState *st) {
    const int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l >= m.layers) return;
    Layer &L = layers[l];
    const int pos = st->position - 1;  // the token the step just processed
    L.due = 0;
    if (pos < 0 || pos == L.last_pos) return;
    L.last_pos = pos;
    if (!m.lighting) {
        if (pos % m.chunk == m.chunk - 1 && *L.relay_count + m.slots <= L.relay_cap) {
            L.due = 1;
            L.relay_base = *L.relay_count;
            *L.relay_count += m.slots;  // read by the next step, after the rows are written
        }
        return;
    }
    // FlashLighting: the row at position pos - window left the window at this step
    // (it was copied aside after the step before)
    const int ms = m.memory_slots;
    int size = *L.relay_count;
    const int in = pos & 1, out = in ^ 1;
    L.stash_in = in;
    L.stash_out = out;
    L.absorb_to = -1;
    L.dst = -1;
    if (pos - m.window >= 0 && L.stash_pos[in] == pos - m.window) {
        if (size + 1 <= ms) {  // room: the row joins memory as it is
            L.absorb_to = size;
            L.mem_slot[size] = size;
            L.mem_pos[size] = L.stash_pos[in];
            L.mem_cnt[size] = 1.0f;
            size += 1;
            L.due |= 1;
        } else {
            // memory + the row exceed memory_slots: the two oldest rows of that list merge
            // (model.py:177-186); with one memory slot the second is the leaving row itself
            const int s0 = L.mem_slot[0];
            const bool second_is_stash = ms < 2;
            const int s1 = second_is_stash ? -1 : L.mem_slot[1];
            const float a = L.mem_cnt[0], b = second_is_stash ? 1.0f : L.mem_cnt[1];
            const int p1 = second_is_stash ? L.stash_pos[in] : L.mem_pos[1];
            const float mean = __fdiv_rn(FADD(FMUL(static_cast<float>(L.mem_pos[0]), a), FMUL(static_cast<float>(p1), b)),
                                         FADD(a, b));
            L.src0 = s0;
            L.src1 = s1;
            L.wa = a;
            L.wb = b;
            L.dst = s0;
            L.merged_pos = static_cast<int>(rintf(mean));
            // logical rows: merged, then the rest, then (with two or more slots) the leaving row
            L.mem_pos[0] = L.merged_pos;
            L.mem_cnt[0] = FADD(a, b);
            if (!second_is_stash) {
                for (int i = 1; i + 1 < ms; ++i) {
                    L.mem_slot[i] = L.mem_slot[i + 1];
                    L.mem_pos[i] = L.mem_pos[i + 1];
                    L.mem_cnt[i] = L.mem_cnt[i + 1];
                }
                L.mem_slot[ms - 1] = s1;  // the freed row takes the leaving row
                L.mem_pos[ms - 1] = L.stash_pos[in];
                L.mem_cnt[ms - 1] = 1.0f;
                L.absorb_to = s1;
                L.due |= 1;
            }
            size = ms;
            L.due |= 2;
        }
    }
    *L.relay_count = size;
    // the row that leaves at the next token, before that step overwrites its ring slot
    const int next = pos + 1 - m.window;
    L.stash_pos[out] = next;
    if (next >= 0) L.due |= 4;
}

// ---- FlashLighting: the merged latent, then the copies (grid: blocks x layers) -----------
// The merge reads the two oldest rows before k_aux_move writes the leaving row over
// the second one's freed slot.
__global__ void __launch_bounds__(kThreads) k_aux_merge(Model m, Layer *layers) {
    const Layer &L = layers[blockIdx.y];
    if (!(L.due & 2)) return;
    const int lat = m.latent, stride = gridDim.x * blockDim.x;
    // kernels.cl merge_rows: (a x0 + b x1) / (a + b)
    const float *x0 = L.mem_lat + static_cast<size_t>(L.src0) * lat;
    const float *x1 = L.src1 >= 0 ? L.mem_lat + static_cast<size_t>(L.src1) * lat : L.stash_lat + L.stash_in * lat;
    float *y = L.mem_lat + static_cast<size_t>(L.dst) * lat;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < lat; i += stride)
        y[i] = __fdiv_rn(FADD(FMUL(L.wa, x0[i]), FMUL(L.wb, x1[i])), FADD(L.wa, L.wb));
}

__global__ void __launch_bounds__(kThreads) k_aux_move(Model m, Layer *layers) {
    const Layer &L = layers[blockIdx.y];
    if (!(L.due & 5)) return;
    const int kvw = L.kv_width, lat = m.latent, ms = m.memory_slots, d = m.d, cap = m.window;
    const int in = L.stash_in, out = L.stash_out;
    const int stride = gridDim.x * blockDim.x, t0 = blockIdx.x * blockDim.x + threadIdx.x;
    // the leaving row into its memory row (latent, key, value as they are)
    if (L.due & 1) {
        const int r = L.absorb_to;
        for (int i = t0; i < lat; i += stride) L.mem_lat[static_cast<size_t>(r) * lat + i] = L.stash_lat[in * lat + i];
        for (int i = t0; i < kvw; i += stride) {
            const int g = i / d, j = i % d;
            L.relay_k[(static_cast<size_t>(g) * ms + r) * d + j] = L.stash_k[in * kvw + i];
            L.relay_v[(static_cast<size_t>(g) * ms + r) * d + j] = L.stash_v[in * kvw + i];
        }
    }
    // the row leaving at the next token: its key, value (ring slot) and normalised latent
    if (L.due & 4) {
        const int q = L.stash_pos[out], slot = q % cap;
        for (int i = t0; i < kvw; i += stride) {
            const int g = i / d, j = i % d;
            L.stash_k[out * kvw + i] = L.k_cache[(static_cast<size_t>(g) * cap + slot) * d + j];
            L.stash_v[out * kvw + i] = L.v_cache[(static_cast<size_t>(g) * cap + slot) * d + j];
        }
        if (blockIdx.x == 0) {  // model.py:156: the stored latent is RMSNorm(latent) * latent_norm
            __shared__ float scale;
            const float *raw = L.lat_ring + static_cast<size_t>(slot) * lat;
            if (threadIdx.x == 0) scale = rms_scale(raw, lat, m.norm_eps);
            __syncthreads();
            for (int i = threadIdx.x; i < lat; i += blockDim.x)
                L.stash_lat[out * lat + i] = FMUL(FMUL(raw[i], scale), load_weight(L.latent_norm, L.latent_norm_dt, i));
        }
    }
}

// One warp per output row r of W [rows][n] against x (n floats): W[r] . x, FMA in column order.
__device__ __forceinline__ float warp_row_dot(const void *w, int dt, int r, const float *x, int n) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    for (int j = lane; j < n; j += 32) acc = fmaf(load_weight(w, dt, static_cast<size_t>(r) * n + j), x[j], acc);
    return warp_sum(acc);
}

// Key (normalised, rotated at `position`) and value of one input row for KV head g,
// written to relay row `row`: block = (head g, key or value), the row's input staged.
__device__ void project_row(const Model &m, const Layer &L, const float *x, int n, int g, bool key, float position,
                            int row) {
    __shared__ float xs[4096];
    __shared__ float out[128];
    __shared__ float scale;
    const int d = m.d, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int j = threadIdx.x; j < n; j += blockDim.x) xs[j] = x[j];
    __syncthreads();
    const void *w = key ? L.wk : L.wv;
    for (int r = warp; r < d; r += nw) {
        const float v = warp_row_dot(w, L.w_dt, g * d + r, xs, n);
        if (lane == 0) out[r] = v;
    }
    __syncthreads();
    float *dst = (key ? L.relay_k : L.relay_v) + (static_cast<size_t>(g) * L.relay_cap + row) * d;
    if (!key) {
        for (int j = threadIdx.x; j < d; j += blockDim.x) dst[j] = out[j];
        return;
    }
    // k_norm (eps norm_eps), then RoPE at the row's position (kernels.cl:30-44)
    if (threadIdx.x == 0) scale = rms_scale(out, d, m.norm_eps);
    __syncthreads();
    const int half = d / 2;
    for (int p = threadIdx.x; p < half; p += blockDim.x) {
        const int j = m.split_half ? p : 2 * p, k = m.split_half ? p + half : 2 * p + 1;
        const float u = FMUL(FMUL(out[j], scale), load_weight(L.k_norm, L.k_norm_dt, j));
        const float v = FMUL(FMUL(out[k], scale), load_weight(L.k_norm, L.k_norm_dt, k));
        const float angle = FMUL(position, m.inv_freq[p]);
        const float cs = cosf(angle), sn = sinf(angle);
        dst[j] = __fsub_rn(FMUL(u, cs), FMUL(v, sn));
        dst[k] = FADD(FMUL(u, sn), FMUL(v, cs));
    }
}

// FlashLighting: the merged row's key and value (grid: layers x 2 kv_heads).
__global__ void __launch_bounds__(kThreads) k_aux_merged_kv(Model m, Layer *layers) {
    const Layer &L = layers[blockIdx.y];
    if (!(L.due & 2) || static_cast<int>(blockIdx.x >> 1) >= L.kv_heads) return;
    const int g = blockIdx.x >> 1;
    project_row(m, L, L.mem_lat + static_cast<size_t>(L.dst) * m.latent, m.latent, g, (blockIdx.x & 1) == 0,
                static_cast<float>(L.merged_pos), L.dst);
}

// ---- flashnano-1.6 pooling --------------------------------------------------------------
// Block t: the chunk's input t normalised (a_norm), its score against every relay query
// (kernels.cl pool_scores: dot / sqrt(hidden)).
__global__ void __launch_bounds__(kThreads) k_cbr_scores(Model m, Layer *layers) {
    const Layer &L = layers[blockIdx.y];
    if (!L.due) return;
    const int t = blockIdx.x, h = m.hidden;
    const float *x = L.pending + static_cast<size_t>(t) * h;
    float *u = L.u + static_cast<size_t>(t) * h;
    __shared__ float scale;
    if (threadIdx.x == 0) scale = rms_scale(x, h, m.norm_eps);
    __syncthreads();
    for (int j = threadIdx.x; j < h; j += blockDim.x) u[j] = FMUL(FMUL(x[j], scale), load_weight(L.a_norm, L.a_norm_dt, j));
    __syncthreads();
    for (int s = threadIdx.x; s < m.slots; s += blockDim.x) {  // kernels.cl pool_scores: a serial dot
        const float *q = L.queries + static_cast<size_t>(s) * h;
        float v = 0.f;
        for (int j = 0; j < h; ++j) v = FADD(v, FMUL(u[j], q[j]));
        L.scores[static_cast<size_t>(s) * m.chunk + t] = __fdiv_rn(v, __fsqrt_rn(static_cast<float>(h)));
    }
}

// Block s: softmax over the chunk (kernels.cl:76-84), the pooled row and its
// rounded anchor (kernels.cl pool_mix), positions start .. start + chunk - 1.
__global__ void __launch_bounds__(kThreads) k_cbr_pool(Model m, Layer *layers, const StepState *st) {
    Layer &L = layers[blockIdx.y];
    if (!L.due) return;
    const int s = blockIdx.x, C = m.chunk, h = m.hidden;
    extern __shared__ float p[];  // [chunk]
    if (threadIdx.x == 0) {  // kernels.cl softmax, then pool_mix's anchor: serial sums
        const float *x = L.scores + static_cast<size_t>(s) * C;
        float mx = -INFINITY;
        for (int t = 0; t < C; ++t) mx = fmaxf(mx, x[t]);
        float den = 0.f;
        for (int t = 0; t < C; ++t) den = FADD(den, expf(__fsub_rn(x[t], mx)));
        float pos = 0.f;
        const int start = st->position - C;  // the chunk's first position
        for (int t = 0; t < C; ++t) {
            p[t] = __fdiv_rn(expf(__fsub_rn(x[t], mx)), den);
            pos = FADD(pos, FMUL(p[t], static_cast<float>(start + t)));
        }
        L.anchors[s] = rintf(pos);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < h; j += blockDim.x) {
        float v = 0.f;
        for (int t = 0; t < C; ++t) v = FADD(v, FMUL(p[t], L.u[static_cast<size_t>(t) * h + j]));
        L.pooled[static_cast<size_t>(s) * h + j] = v;
    }
}

// Block (slot s, head g, key / value): the relay row's key or value.
__global__ void __launch_bounds__(kThreads) k_cbr_kv(Model m, Layer *layers) {
    const Layer &L = layers[blockIdx.y];
    if (!L.due) return;
    const int s = blockIdx.x / (2 * L.kv_heads), rest = blockIdx.x % (2 * L.kv_heads);
    if (s >= m.slots) return;
    project_row(m, L, L.pooled + static_cast<size_t>(s) * m.hidden, m.hidden, rest >> 1, (rest & 1) == 0,
                L.anchors[s], L.relay_base + s);
}

// rows x n values normalised without a gain (model.py:124: the relay queries,
// RMSNorm(cbr, eps = cbr_norm_eps)), the norm kernel's arithmetic.
__global__ void k_norm_rows(const void *x, int dt, int rows, int n, float eps, float *y) {
    const int r = blockIdx.x;
    if (r >= rows || threadIdx.x != 0) return;
    float ss = 0.f;
    for (int j = 0; j < n; ++j) {
        const float v = load_weight(x, dt, static_cast<size_t>(r) * n + j);
        ss = FADD(ss, FMUL(v, v));
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(FADD(__fdiv_rn(ss, static_cast<float>(n)), eps)));
    for (int j = 0; j < n; ++j) y[static_cast<size_t>(r) * n + j] = FMUL(load_weight(x, dt, static_cast<size_t>(r) * n + j), scale);
}

}  // namespace aux
}  // namespace mr
