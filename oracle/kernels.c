/*
 * CPU oracle: a plain-C restatement of the thirteen OpenCL kernels of the
 * MiracleReasoning token loop (miracle_reasoning/kernels.cl).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA product is
 * compared against; it is never linked into, called by, or shipped with the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load the library built from it.
 *
 * Arithmetic contract (what makes this an oracle rather than "some CPU code"):
 *   - compiled with -ffp-contract=off, so a*b+c is a rounded product followed by
 *     a rounded sum, exactly as `#pragma OPENCL FP_CONTRACT OFF` (kernels.cl:3)
 *     demands of the reference;
 *   - every reduction runs in the reference's serial order (named per kernel);
 *   - transcendentals are single precision libm (sqrtf/expf/sinf/cosf/rintf),
 *     which is what an OpenCL CPU runtime built on the host libm computes.
 *
 * Each entry point takes the NDRange extents first (g0[, g1]) and then the
 * kernel's own arguments in the kernel's order, and evaluates every work item
 * of that NDRange, applying the kernel's own early-return bounds test.  Work
 * items are independent, so the outer loops are OpenMP-parallel; this changes
 * no result.
 */
#include <math.h>
#include <stddef.h>

#define OMP_FOR _Pragma("omp parallel for schedule(static)")

/* kernels.cl:5-17 — four lane-wise partial sums over j = 0,4,8,... in serial
 * order, folded as ((s0+s1)+s2)+s3, then a serial scalar tail. */
void mo_linear(size_t g0, size_t g1, const float *x, const float *w, float *y,
               int rows, int out_dim, int in_dim) {
    long long total = (long long)g0 * (long long)g1;
    OMP_FOR
    for (long long item = 0; item < total; ++item) {
        size_t o = (size_t)(item % (long long)g0), r = (size_t)(item / (long long)g0);
        if (o >= (size_t)out_dim || r >= (size_t)rows) continue;
        const float *xr = x + r * (size_t)in_dim, *wr = w + o * (size_t)in_dim;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        int j = 0;
        for (; j + 3 < in_dim; j += 4) {
            s0 += xr[j] * wr[j];
            s1 += xr[j + 1] * wr[j + 1];
            s2 += xr[j + 2] * wr[j + 2];
            s3 += xr[j + 3] * wr[j + 3];
        }
        float v = ((s0 + s1) + s2) + s3;
        for (; j < in_dim; ++j) v += xr[j] * wr[j];
        y[r * (size_t)out_dim + o] = v;
    }
}

/* kernels.cl:19-28 — serial sum of squares, scale = 1/sqrt(mean+eps),
 * y = (x*scale)*gain, gain taken as 1 when the norm is not affine. */
void mo_rms(size_t g0, const float *x, const float *w, float *y, int rows,
            int width, float eps, int affine) {
    OMP_FOR
    for (long long rr = 0; rr < (long long)g0; ++rr) {
        size_t r = (size_t)rr;
        if (r >= (size_t)rows) continue;
        const float *xr = x + r * (size_t)width;
        float v = 0.0f;
        for (int j = 0; j < width; ++j) { float a = xr[j]; v += a * a; }
        float scale = 1.0f / sqrtf(v / (float)width + eps);
        for (int j = 0; j < width; ++j)
            y[r * (size_t)width + j] = xr[j] * scale * (affine ? w[j] : 1.0f);
    }
}

/* kernels.cl:30-44 — one work item per rotated pair.  Pair (2p,2p+1) when
 * interleaved, (p,p+dim/2) when split-half; angle = pos[row]*freq[p]. */
void mo_rope(size_t g0, const float *x, const float *freq, const float *pos,
             float *y, int rows, int heads, int dim, int split_half) {
    int half = dim / 2;
    size_t limit = (size_t)rows * (size_t)heads * (size_t)half;
    OMP_FOR
    for (long long ii = 0; ii < (long long)g0; ++ii) {
        size_t i = (size_t)ii;
        if (i >= limit) continue;
        int p = (int)(i % (size_t)half);
        size_t head_row = i / (size_t)half, base = head_row * (size_t)dim;
        float angle = pos[head_row / (size_t)heads] * freq[p];
        float c = cosf(angle), s = sinf(angle);
        int j = split_half ? p : 2 * p;
        int k = split_half ? p + half : 2 * p + 1;
        float u = x[base + j], v = x[base + k];
        y[base + j] = u * c - v * s;
        y[base + k] = u * s + v * c;
    }
}

/* kernels.cl:46-50 */
void mo_swiglu(size_t g0, const float *g, const float *u, float *y, int n) {
    OMP_FOR
    for (long long i = 0; i < (long long)g0; ++i)
        if (i < n) y[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

/* kernels.cl:52-56 */
void mo_axpy(size_t g0, const float *x, const float *yv, float *z, int n, float scale) {
    OMP_FOR
    for (long long i = 0; i < (long long)g0; ++i)
        if (i < n) z[i] = x[i] + scale * yv[i];
}

static size_t ring_row(size_t t, int length, int start, int capacity) {
    return t < (size_t)length ? ((size_t)start + t) % (size_t)capacity : t - (size_t)length;
}

/* kernels.cl:58-73 — logical ring order [start, start+length) modulo the
 * capacity, then extra rows; serial dot product, divided by sqrt(dim). */
void mo_scores(size_t g0, size_t g1, const float *q, const float *k,
               const float *extra_k, float *s, int heads, int kv_heads, int dim,
               int capacity, int start, int length, int extra_length) {
    long long total_items = (long long)g0 * (long long)g1;
    int total = length + extra_length;
    OMP_FOR
    for (long long item = 0; item < total_items; ++item) {
        size_t t = (size_t)(item % (long long)g0), h = (size_t)(item / (long long)g0);
        if (t >= (size_t)total || h >= (size_t)heads) continue;
        int kh = (int)h / (heads / kv_heads);
        size_t kb = ring_row(t, length, start, capacity) * (size_t)kv_heads * dim + (size_t)kh * dim;
        const float *src = t < (size_t)length ? k : extra_k;
        float v = 0.0f;
        for (int j = 0; j < dim; ++j) v += q[h * dim + j] * src[kb + j];
        s[h * (size_t)total + t] = v / sqrtf((float)dim);
    }
}

/* kernels.cl:75-84 — row max, serial sum of exp(x-m), then exp(x-m)/denom. */
void mo_softmax(size_t g0, const float *x, float *y, int rows, int width) {
    OMP_FOR
    for (long long rr = 0; rr < (long long)g0; ++rr) {
        size_t r = (size_t)rr;
        if (r >= (size_t)rows) continue;
        const float *xr = x + r * (size_t)width;
        float m = -INFINITY;
        for (int j = 0; j < width; ++j) m = fmaxf(m, xr[j]);
        float denom = 0.0f;
        for (int j = 0; j < width; ++j) denom += expf(xr[j] - m);
        for (int j = 0; j < width; ++j) y[r * (size_t)width + j] = expf(xr[j] - m) / denom;
    }
}

/* kernels.cl:86-91 — float position compared against the integer horizon. */
void mo_latent_mask(size_t g0, size_t g1, float *scores, const float *positions,
                    int heads, int length, int memory, int earliest) {
    long long total = (long long)g0 * (long long)g1;
    OMP_FOR
    for (long long item = 0; item < total; ++item) {
        size_t t = (size_t)(item % (long long)g0), h = (size_t)(item / (long long)g0);
        if (t < (size_t)length && h < (size_t)heads && t >= (size_t)memory &&
            positions[t] < (float)earliest)
            scores[h * (size_t)length + t] = -INFINITY;
    }
}

/* kernels.cl:93-107 — serial sum over t of p[h,t]*v[row(t),kh,j]. */
void mo_mix(size_t g0, const float *p, const float *v, const float *extra_v, float *y,
            int heads, int kv_heads, int dim, int capacity, int start, int length,
            int extra_length) {
    size_t limit = (size_t)heads * (size_t)dim;
    OMP_FOR
    for (long long ii = 0; ii < (long long)g0; ++ii) {
        size_t i = (size_t)ii;
        if (i >= limit) continue;
        int h = (int)(i / (size_t)dim), j = (int)(i % (size_t)dim);
        int kh = h / (heads / kv_heads), total = length + extra_length;
        float acc = 0.0f;
        for (int t = 0; t < total; ++t) {
            size_t vb = ring_row((size_t)t, length, start, capacity) * (size_t)kv_heads * dim +
                        (size_t)kh * dim + j;
            acc += p[(size_t)h * total + t] * (t < length ? v[vb] : extra_v[vb]);
        }
        y[i] = acc;
    }
}

/* kernels.cl:109-117 — CBR pooling scores u_t . q_m / sqrt(width). */
void mo_pool_scores(size_t g0, size_t g1, const float *u, const float *q, float *s,
                    int tokens, int slots, int width) {
    long long total = (long long)g0 * (long long)g1;
    OMP_FOR
    for (long long item = 0; item < total; ++item) {
        size_t t = (size_t)(item % (long long)g0), m = (size_t)(item / (long long)g0);
        if (t >= (size_t)tokens || m >= (size_t)slots) continue;
        float v = 0.0f;
        for (int j = 0; j < width; ++j) v += u[t * width + j] * q[m * width + j];
        s[m * (size_t)tokens + t] = v / sqrtf((float)width);
    }
}

/* kernels.cl:119-130 — pooled rows and rounded probability-weighted anchors. */
void mo_pool_mix(size_t g0, size_t g1, const float *u, const float *p, float *z,
                 float *anchors, int tokens, int slots, int width, int start_position) {
    long long total = (long long)g0 * (long long)g1;
    OMP_FOR
    for (long long item = 0; item < total; ++item) {
        size_t j = (size_t)(item % (long long)g0), m = (size_t)(item / (long long)g0);
        if (j >= (size_t)width || m >= (size_t)slots) continue;
        float v = 0.0f, pos = 0.0f;
        for (int t = 0; t < tokens; ++t) {
            float wt = p[m * (size_t)tokens + t];
            v += wt * u[(size_t)t * width + j];
            pos += wt * (float)(start_position + t);
        }
        z[m * (size_t)width + j] = v;
        if (j == 0) anchors[m] = rintf(pos);
    }
}

/* kernels.cl:132-137 */
void mo_merge_rows(size_t g0, const float *x, float *y, int width, float a, float b) {
    OMP_FOR
    for (long long j = 0; j < (long long)g0; ++j)
        if (j < width) y[j] = (a * x[j] + b * x[width + j]) / (a + b);
}

/* kernels.cl:139-148 — serial mean of each block of rows; the last block is the
 * partial prefix. */
void mo_block_means(size_t g0, size_t g1, const float *x, float *y, int length,
                    int width, int block) {
    long long total = (long long)g0 * (long long)g1;
    OMP_FOR
    for (long long item = 0; item < total; ++item) {
        size_t j = (size_t)(item % (long long)g0), b = (size_t)(item / (long long)g0);
        int start = (int)b * block, stop = start + block < length ? start + block : length;
        if (j >= (size_t)width || start >= length) continue;
        float v = 0.0f;
        for (int t = start; t < stop; ++t) v += x[(size_t)t * width + j];
        y[b * (size_t)width + j] = v / (float)(stop - start);
    }
}
