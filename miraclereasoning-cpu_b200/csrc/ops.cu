// One CUDA kernel per reference kernel (miracle_reasoning/kernels.cl), behind
// the mr_op_* entry points.  They serve the reference backend's op surface
// (opencl.py:219-300), so the reference's own call sites and kernel tests run
// on the GPU unchanged; the decode hot path uses the fused engine instead.
//
// Arithmetic follows kernels.cl work item by work item: the same reduction
// order, and every product and sum rounded separately (__fmul_rn/__fadd_rn:
// the reference compiles with FP_CONTRACT OFF, kernels.cl:3).  Division and
// square root are IEEE; exp/sin/cos are CUDA's full-range single-precision
// functions (a few ulp from the host libm), never the __ intrinsics.
//
// Every entry point checks each buffer extent the kernel can touch before it
// launches, so a bad argument is an MR_ERR_ARGUMENT, never a device fault.
#include <algorithm>
#include <climits>

#include "common.cuh"

namespace {

constexpr int kThreads = 256;

inline unsigned blocks_for(size_t items) {
    return static_cast<unsigned>((items + kThreads - 1) / kThreads);
}

#define FADD __fadd_rn
#define FMUL __fmul_rn

__global__ void k_linear(size_t g0, size_t g1, const float *x, const float *w, float *y, int rows,
                         int out_dim, int in_dim) {
    size_t item = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (item >= g0 * g1) return;
    size_t o = item % g0, r = item / g0;
    if (o >= (size_t)out_dim || r >= (size_t)rows) return;
    const float *xr = x + r * in_dim, *wr = w + o * in_dim;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int j = 0;
    for (; j + 3 < in_dim; j += 4) {
        s0 = FADD(s0, FMUL(xr[j], wr[j]));
        s1 = FADD(s1, FMUL(xr[j + 1], wr[j + 1]));
        s2 = FADD(s2, FMUL(xr[j + 2], wr[j + 2]));
        s3 = FADD(s3, FMUL(xr[j + 3], wr[j + 3]));
    }
    float v = FADD(FADD(FADD(s0, s1), s2), s3);
    for (; j < in_dim; ++j) v = FADD(v, FMUL(xr[j], wr[j]));
    y[r * out_dim + o] = v;
}

__global__ void k_rms(size_t g0, const float *x, const float *w, float *y, int rows, int width, float eps,
                      int affine) {
    size_t r = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (r >= g0 || r >= (size_t)rows) return;
    const float *xr = x + r * width;
    float v = 0.f;
    for (int j = 0; j < width; ++j) v = FADD(v, FMUL(xr[j], xr[j]));
    float scale = __fdiv_rn(1.0f, __fsqrt_rn(FADD(__fdiv_rn(v, (float)width), eps)));
    for (int j = 0; j < width; ++j) y[r * width + j] = FMUL(FMUL(xr[j], scale), affine ? w[j] : 1.0f);
}

__global__ void k_rope(size_t g0, const float *x, const float *freq, const float *pos, float *y, int rows,
                       int heads, int dim, int split_half) {
    size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    int half = dim / 2;
    if (i >= g0 || i >= (size_t)rows * heads * half) return;
    int p = i % half;
    size_t head_row = i / half, base = head_row * dim;
    float angle = FMUL(pos[head_row / heads], freq[p]);
    float c = cosf(angle), s = sinf(angle);
    int j = split_half ? p : 2 * p, k = split_half ? p + half : 2 * p + 1;
    float u = x[base + j], v = x[base + k];
    y[base + j] = __fsub_rn(FMUL(u, c), FMUL(v, s));
    y[base + k] = FADD(FMUL(u, s), FMUL(v, c));
}

__global__ void k_swiglu(size_t g0, const float *g, const float *u, float *y, int n) {
    size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (i >= g0 || i >= (size_t)n) return;
    y[i] = FMUL(__fdiv_rn(g[i], FADD(1.0f, expf(-g[i]))), u[i]);
}

__global__ void k_axpy(size_t g0, const float *x, const float *yv, float *z, int n, float scale) {
    size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (i >= g0 || i >= (size_t)n) return;
    z[i] = FADD(x[i], FMUL(scale, yv[i]));
}

__device__ __forceinline__ size_t ring_row(size_t t, int length, int start, int capacity) {
    return t < (size_t)length ? ((size_t)start + t) % (size_t)capacity : t - (size_t)length;
}

__global__ void k_scores(size_t g0, size_t g1, const float *q, const float *k, const float *extra_k, float *s,
                         int heads, int kv_heads, int dim, int capacity, int start, int length,
                         int extra_length) {
    size_t item = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (item >= g0 * g1) return;
    size_t t = item % g0, h = item / g0;
    int total = length + extra_length;
    if (t >= (size_t)total || h >= (size_t)heads) return;
    int kh = (int)h / (heads / kv_heads);
    size_t kb = ring_row(t, length, start, capacity) * kv_heads * dim + (size_t)kh * dim;
    const float *src = t < (size_t)length ? k : extra_k;
    float v = 0.f;
    for (int j = 0; j < dim; ++j) v = FADD(v, FMUL(q[h * dim + j], src[kb + j]));
    s[h * total + t] = __fdiv_rn(v, __fsqrt_rn((float)dim));
}

__global__ void k_softmax(size_t g0, const float *x, float *y, int rows, int width) {
    size_t r = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (r >= g0 || r >= (size_t)rows) return;
    const float *xr = x + r * width;
    float m = -INFINITY;
    for (int j = 0; j < width; ++j) m = fmaxf(m, xr[j]);
    float denom = 0.f;
    for (int j = 0; j < width; ++j) denom = FADD(denom, expf(__fsub_rn(xr[j], m)));
    for (int j = 0; j < width; ++j) y[r * width + j] = __fdiv_rn(expf(__fsub_rn(xr[j], m)), denom);
}

__global__ void k_latent_mask(size_t g0, size_t g1, float *scores, const float *positions, int heads,
                              int length, int memory, int earliest) {
    size_t item = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (item >= g0 * g1) return;
    size_t t = item % g0, h = item / g0;
    if (t < (size_t)length && h < (size_t)heads && t >= (size_t)memory && positions[t] < (float)earliest)
        scores[h * length + t] = -INFINITY;
}

__global__ void k_mix(size_t g0, const float *p, const float *v, const float *extra_v, float *y, int heads,
                      int kv_heads, int dim, int capacity, int start, int length, int extra_length) {
    size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (i >= g0 || i >= (size_t)heads * dim) return;
    int h = i / dim, j = i % dim, kh = h / (heads / kv_heads), total = length + extra_length;
    float acc = 0.f;
    for (int t = 0; t < total; ++t) {
        size_t vb = ring_row(t, length, start, capacity) * kv_heads * dim + (size_t)kh * dim + j;
        acc = FADD(acc, FMUL(p[(size_t)h * total + t], t < length ? v[vb] : extra_v[vb]));
    }
    y[i] = acc;
}

__global__ void k_pool_scores(size_t g0, size_t g1, const float *u, const float *q, float *s, int tokens,
                              int slots, int width) {
    size_t item = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (item >= g0 * g1) return;
    size_t t = item % g0, m = item / g0;
    if (t >= (size_t)tokens || m >= (size_t)slots) return;
    float v = 0.f;
    for (int j = 0; j < width; ++j) v = FADD(v, FMUL(u[t * width + j], q[m * width + j]));
    s[m * tokens + t] = __fdiv_rn(v, __fsqrt_rn((float)width));
}

__global__ void k_pool_mix(size_t g0, size_t g1, const float *u, const float *p, float *z, float *anchors,
                           int tokens, int slots, int width, int start_position) {
    size_t item = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (item >= g0 * g1) return;
    size_t j = item % g0, m = item / g0;
    if (j >= (size_t)width || m >= (size_t)slots) return;
    float v = 0.f, pos = 0.f;
    for (int t = 0; t < tokens; ++t) {
        float w = p[m * tokens + t];
        v = FADD(v, FMUL(w, u[(size_t)t * width + j]));
        pos = FADD(pos, FMUL(w, (float)(start_position + t)));
    }
    z[m * width + j] = v;
    if (j == 0) anchors[m] = rintf(pos);
}

__global__ void k_merge_rows(size_t g0, const float *x, float *y, int width, float a, float b) {
    size_t j = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (j >= g0 || j >= (size_t)width) return;
    y[j] = __fdiv_rn(FADD(FMUL(a, x[j]), FMUL(b, x[width + j])), FADD(a, b));
}

__global__ void k_block_means(size_t g0, size_t g1, const float *x, float *y, int length, int width,
                              int block) {
    size_t item = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (item >= g0 * g1) return;
    size_t j = item % g0, b = item / g0;
    int start = (int)b * block, stop = min(start + block, length);
    if (j >= (size_t)width || start >= length) return;
    float v = 0.f;
    for (int t = start; t < stop; ++t) v = FADD(v, x[(size_t)t * width + j]);
    y[b * width + j] = __fdiv_rn(v, (float)(stop - start));
}

// ---- argument checks -----------------------------------------------------------
struct Check {
    mr_context *ctx;
    int rc = MR_OK;
    bool buf(const mr_buffer *b, size_t need, const char *what) {
        if (rc) return false;
        if (!b) {
            rc = mr::set_error(MR_ERR_ARGUMENT, "%s buffer is NULL", what);
            return false;
        }
        if (b->ctx != ctx) {
            rc = mr::set_error(MR_ERR_ARGUMENT, "Tensors belong to different CUDA contexts");
            return false;
        }
        if (need > b->count) {
            rc = mr::set_error(MR_ERR_ARGUMENT, "%s needs %zu floats, buffer has %zu", what, need, b->count);
            return false;
        }
        return true;
    }
    bool nonneg(long long v, const char *what) {
        if (!rc && v < 0) rc = mr::set_error(MR_ERR_ARGUMENT, "%s must be non-negative", what);
        return !rc;
    }
};

inline size_t lo(size_t a, long long b) { return std::min(a, static_cast<size_t>(b < 0 ? 0 : b)); }

int launch_done(const char *name) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return mr::cuda_error(err, name);
    return MR_OK;
}

#define BEGIN_OP(ctx)                                                       \
    if (!(ctx)) return mr::set_error(MR_ERR_ARGUMENT, "ctx is NULL");       \
    Check ck{ctx};                                                          \
    MR_CUDA_TRY(cudaSetDevice((ctx)->device))

int check_attention_geometry(Check &ck, int heads, int kv_heads, int dim, int capacity, int start, int length,
                             int extra_length) {
    ck.nonneg(heads, "heads") && ck.nonneg(dim, "dim") && ck.nonneg(length, "length") &&
        ck.nonneg(extra_length, "extra_length") && ck.nonneg(start, "start");
    if (!ck.rc && static_cast<long long>(length) + extra_length > INT_MAX)
        ck.rc = mr::set_error(MR_ERR_ARGUMENT, "length + extra_length exceeds the int range");
    if (!ck.rc && (kv_heads <= 0 || heads < kv_heads))
        ck.rc = mr::set_error(MR_ERR_ARGUMENT, "kv_heads must be in [1, heads]");
    if (!ck.rc && length > 0 && capacity <= 0) ck.rc = mr::set_error(MR_ERR_ARGUMENT, "capacity must be positive");
    return ck.rc;
}

}  // namespace

extern "C" {

int mr_op_linear(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *x, const mr_buffer *w,
                 mr_buffer *y, int rows, int out_dim, int in_dim) {
    BEGIN_OP(ctx);
    ck.nonneg(rows, "rows") && ck.nonneg(out_dim, "out_dim") && ck.nonneg(in_dim, "in_dim");
    size_t r = lo(g1, rows), o = lo(g0, out_dim);
    if (r && o) {
        ck.buf(x, r * in_dim, "x") && ck.buf(w, o * in_dim, "w") && ck.buf(y, (r - 1) * (size_t)out_dim + o, "y");
    }
    if (ck.rc) return ck.rc;
    if (!r || !o) return MR_OK;
    k_linear<<<blocks_for(g0 * g1), kThreads, 0, ctx->stream>>>(g0, g1, x->ptr, w->ptr, y->ptr, rows, out_dim,
                                                                in_dim);
    return launch_done("linear");
}

int mr_op_rms(mr_context *ctx, size_t g0, const mr_buffer *x, const mr_buffer *w, mr_buffer *y, int rows,
              int width, float eps, int affine) {
    BEGIN_OP(ctx);
    ck.nonneg(rows, "rows") && ck.nonneg(width, "width");
    size_t r = lo(g0, rows);
    if (r) ck.buf(x, r * width, "x") && ck.buf(y, r * width, "y") && (!affine || ck.buf(w, width, "w"));
    if (ck.rc) return ck.rc;
    if (!r) return MR_OK;
    k_rms<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, x->ptr, affine ? w->ptr : x->ptr, y->ptr, rows, width,
                                                        eps, affine);
    return launch_done("rms");
}

int mr_op_rope(mr_context *ctx, size_t g0, const mr_buffer *x, const mr_buffer *freq, const mr_buffer *pos,
               mr_buffer *y, int rows, int heads, int dim, int split_half) {
    BEGIN_OP(ctx);
    ck.nonneg(rows, "rows") && ck.nonneg(heads, "heads") && ck.nonneg(dim, "dim");
    size_t items = dim >= 2 ? lo(g0, (long long)rows * heads * (dim / 2)) : 0;
    if (items) {
        size_t head_rows = (items + dim / 2 - 1) / (dim / 2);
        size_t pos_rows = (head_rows + heads - 1) / heads;
        ck.buf(x, head_rows * dim, "x") && ck.buf(y, head_rows * dim, "y") && ck.buf(freq, dim / 2, "freq") &&
            ck.buf(pos, pos_rows, "positions");
    }
    if (ck.rc) return ck.rc;
    if (!items) return MR_OK;
    k_rope<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, x->ptr, freq->ptr, pos->ptr, y->ptr, rows, heads, dim,
                                                         split_half);
    return launch_done("rope");
}

int mr_op_swiglu(mr_context *ctx, size_t g0, const mr_buffer *g, const mr_buffer *u, mr_buffer *y, int n) {
    BEGIN_OP(ctx);
    size_t m = lo(g0, n);
    if (m) ck.buf(g, m, "gate") && ck.buf(u, m, "up") && ck.buf(y, m, "y");
    if (ck.rc) return ck.rc;
    if (!m) return MR_OK;
    k_swiglu<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, g->ptr, u->ptr, y->ptr, n);
    return launch_done("swiglu");
}

int mr_op_axpy(mr_context *ctx, size_t g0, const mr_buffer *x, const mr_buffer *y, mr_buffer *z, int n,
               float scale) {
    BEGIN_OP(ctx);
    size_t m = lo(g0, n);
    if (m) ck.buf(x, m, "x") && ck.buf(y, m, "y") && ck.buf(z, m, "z");
    if (ck.rc) return ck.rc;
    if (!m) return MR_OK;
    k_axpy<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, x->ptr, y->ptr, z->ptr, n, scale);
    return launch_done("axpy");
}

int mr_op_scores(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *q, const mr_buffer *k,
                 const mr_buffer *extra_k, mr_buffer *s, int heads, int kv_heads, int dim, int capacity,
                 int start, int length, int extra_length) {
    BEGIN_OP(ctx);
    if (check_attention_geometry(ck, heads, kv_heads, dim, capacity, start, length, extra_length)) return ck.rc;
    int total = length + extra_length;
    size_t t = lo(g0, total), h = lo(g1, heads);
    if (t && h) {
        size_t row = (size_t)kv_heads * dim;
        // rows [start, start + length) mod capacity: 64-bit, so a start near INT_MAX cannot wrap
        const long long ring_end = static_cast<long long>(start) + length;
        size_t ring_rows = ring_end > capacity ? (size_t)capacity : (size_t)ring_end;
        ck.buf(q, h * dim, "q") && ck.buf(s, (h - 1) * (size_t)total + t, "scores") &&
            (length == 0 || ck.buf(k, ring_rows * row, "keys")) &&
            (t <= (size_t)length || ck.buf(extra_k, (t - length) * row, "extra keys"));
    }
    if (ck.rc) return ck.rc;
    if (!t || !h) return MR_OK;
    k_scores<<<blocks_for(g0 * g1), kThreads, 0, ctx->stream>>>(
        g0, g1, q->ptr, length ? k->ptr : nullptr, extra_k ? extra_k->ptr : nullptr, s->ptr, heads, kv_heads, dim,
        capacity, start, length, extra_length);
    return launch_done("scores");
}

int mr_op_softmax(mr_context *ctx, size_t g0, const mr_buffer *x, mr_buffer *y, int rows, int width) {
    BEGIN_OP(ctx);
    ck.nonneg(rows, "rows") && ck.nonneg(width, "width");
    size_t r = lo(g0, rows);
    if (r) ck.buf(x, r * width, "x") && ck.buf(y, r * width, "y");
    if (ck.rc) return ck.rc;
    if (!r) return MR_OK;
    k_softmax<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, x->ptr, y->ptr, rows, width);
    return launch_done("softmax");
}

int mr_op_latent_mask(mr_context *ctx, size_t g0, size_t g1, mr_buffer *scores, const mr_buffer *positions,
                      int heads, int length, int memory, int earliest) {
    BEGIN_OP(ctx);
    ck.nonneg(heads, "heads") && ck.nonneg(length, "length");
    size_t t = lo(g0, length), h = lo(g1, heads);
    if (t && h) ck.buf(scores, (h - 1) * (size_t)length + t, "scores") && ck.buf(positions, t, "positions");
    if (ck.rc) return ck.rc;
    if (!t || !h) return MR_OK;
    k_latent_mask<<<blocks_for(g0 * g1), kThreads, 0, ctx->stream>>>(g0, g1, scores->ptr, positions->ptr, heads,
                                                                     length, memory, earliest);
    return launch_done("latent_mask");
}

int mr_op_mix(mr_context *ctx, size_t g0, const mr_buffer *p, const mr_buffer *v, const mr_buffer *extra_v,
              mr_buffer *y, int heads, int kv_heads, int dim, int capacity, int start, int length,
              int extra_length) {
    BEGIN_OP(ctx);
    if (check_attention_geometry(ck, heads, kv_heads, dim, capacity, start, length, extra_length)) return ck.rc;
    size_t items = lo(g0, (long long)heads * dim);
    if (items) {
        size_t row = (size_t)kv_heads * dim, total = length + extra_length;
        size_t used_heads = (items + dim - 1) / dim;
        // rows [start, start + length) mod capacity: 64-bit, so a start near INT_MAX cannot wrap
        const long long ring_end = static_cast<long long>(start) + length;
        size_t ring_rows = ring_end > capacity ? (size_t)capacity : (size_t)ring_end;
        ck.buf(p, used_heads * total, "probabilities") && ck.buf(y, items, "y") &&
            (length == 0 || ck.buf(v, ring_rows * row, "values")) &&
            (extra_length == 0 || ck.buf(extra_v, (size_t)extra_length * row, "extra values"));
    }
    if (ck.rc) return ck.rc;
    if (!items) return MR_OK;
    k_mix<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, p->ptr, length ? v->ptr : nullptr,
                                                        extra_v ? extra_v->ptr : nullptr, y->ptr, heads, kv_heads,
                                                        dim, capacity, start, length, extra_length);
    return launch_done("mix");
}

int mr_op_pool_scores(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *u, const mr_buffer *q,
                      mr_buffer *s, int tokens, int slots, int width) {
    BEGIN_OP(ctx);
    ck.nonneg(tokens, "tokens") && ck.nonneg(slots, "slots") && ck.nonneg(width, "width");
    size_t t = lo(g0, tokens), m = lo(g1, slots);
    if (t && m)
        ck.buf(u, t * width, "u") && ck.buf(q, m * width, "queries") && ck.buf(s, (m - 1) * (size_t)tokens + t, "scores");
    if (ck.rc) return ck.rc;
    if (!t || !m) return MR_OK;
    k_pool_scores<<<blocks_for(g0 * g1), kThreads, 0, ctx->stream>>>(g0, g1, u->ptr, q->ptr, s->ptr, tokens, slots,
                                                                     width);
    return launch_done("pool_scores");
}

int mr_op_pool_mix(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *u, const mr_buffer *p, mr_buffer *z,
                   mr_buffer *anchors, int tokens, int slots, int width, int start_position) {
    BEGIN_OP(ctx);
    ck.nonneg(tokens, "tokens") && ck.nonneg(slots, "slots") && ck.nonneg(width, "width");
    size_t j = lo(g0, width), m = lo(g1, slots);
    if (j && m)
        ck.buf(u, (size_t)tokens * width, "u") && ck.buf(p, m * (size_t)tokens, "probabilities") &&
            ck.buf(z, (m - 1) * (size_t)width + j, "pooled") && ck.buf(anchors, m, "anchors");
    if (ck.rc) return ck.rc;
    if (!j || !m) return MR_OK;
    k_pool_mix<<<blocks_for(g0 * g1), kThreads, 0, ctx->stream>>>(g0, g1, u->ptr, p->ptr, z->ptr, anchors->ptr, tokens,
                                                                  slots, width, start_position);
    return launch_done("pool_mix");
}

int mr_op_merge_rows(mr_context *ctx, size_t g0, const mr_buffer *x, mr_buffer *y, int width, float a, float b) {
    BEGIN_OP(ctx);
    ck.nonneg(width, "width");
    size_t j = lo(g0, width);
    if (j) ck.buf(x, (size_t)width + j, "x") && ck.buf(y, j, "y");
    if (ck.rc) return ck.rc;
    if (!j) return MR_OK;
    k_merge_rows<<<blocks_for(g0), kThreads, 0, ctx->stream>>>(g0, x->ptr, y->ptr, width, a, b);
    return launch_done("merge_rows");
}

int mr_op_block_means(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *x, mr_buffer *y, int length,
                      int width, int block) {
    BEGIN_OP(ctx);
    ck.nonneg(length, "length") && ck.nonneg(width, "width");
    if (!ck.rc && block <= 0) ck.rc = mr::set_error(MR_ERR_ARGUMENT, "block must be positive");
    if (ck.rc) return ck.rc;
    size_t j = lo(g0, width);
    size_t blocks = lo(g1, (length + block - 1) / block);
    if (j && blocks) ck.buf(x, (size_t)length * width, "x") && ck.buf(y, (blocks - 1) * (size_t)width + j, "y");
    if (ck.rc) return ck.rc;
    if (!j || !blocks) return MR_OK;
    k_block_means<<<blocks_for(g0 * g1), kThreads, 0, ctx->stream>>>(g0, g1, x->ptr, y->ptr, length, width, block);
    return launch_done("block_means");
}

}  // extern "C"
