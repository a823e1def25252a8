// Host build of the reference's own OpenCL kernels (TEST INFRASTRUCTURE ONLY).
//
// The reference's miracle_reasoning/kernels.cl is compiled UNMODIFIED, from
// where it lies, as C++ inside namespace refcl.  The few lines before the
// #include supply the OpenCL C built-ins that file uses (address-space
// qualifiers, float4 with lane-wise * and +=, vload4, get_global_id and the
// single-precision math functions).  Each extern "C" wrapper below evaluates
// one NDRange: it walks every global id, publishes it through get_global_id,
// and calls the reference kernel, which applies its own bounds test.
//
// The output library (oracle/_ref/libref_kernels.so) is used in two places
// only: to pin the plain-C restatement in oracle/kernels.c bit for bit, and as
// the timed CPU baseline ("kind": "reference") in bench.py.  The path of
// kernels.cl is passed at build time as REF_KERNELS_CL.
#include <algorithm>
#include <cmath>
#include <cstddef>

namespace refcl {

static thread_local size_t g_global_id[3];
static inline size_t get_global_id(int dim) { return g_global_id[dim]; }

struct float4 {
    float x, y, z, w;
    float4() : x(0), y(0), z(0), w(0) {}
    explicit float4(float s) : x(s), y(s), z(s), w(s) {}
    float4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
};
static inline float4 operator*(const float4 &a, const float4 &b) {
    return float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}
static inline float4 &operator+=(float4 &a, const float4 &b) {
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    return a;
}
static inline float4 vload4(size_t offset, const float *p) {
    p += offset * 4;
    return float4(p[0], p[1], p[2], p[3]);
}
using std::cos;
using std::exp;
using std::fmax;
using std::min;
using std::rint;
using std::sin;
using std::sqrt;

#define __kernel
#define __global
#include REF_KERNELS_CL
#undef __kernel
#undef __global

}  // namespace refcl

#define RANGE1(g0, call)                                                    \
    _Pragma("omp parallel for schedule(static)")                            \
    for (long long i0 = 0; i0 < (long long)(g0); ++i0) {                    \
        refcl::g_global_id[0] = (size_t)i0;                                 \
        call;                                                               \
    }
#define RANGE2(g0, g1, call)                                                \
    _Pragma("omp parallel for schedule(static)")                            \
    for (long long it = 0; it < (long long)(g0) * (long long)(g1); ++it) {  \
        refcl::g_global_id[0] = (size_t)(it % (long long)(g0));             \
        refcl::g_global_id[1] = (size_t)(it / (long long)(g0));             \
        call;                                                               \
    }

extern "C" {

void ref_linear(size_t g0, size_t g1, const float *x, const float *w, float *y, int rows,
                int out_dim, int in_dim) {
    RANGE2(g0, g1, refcl::linear(x, w, y, rows, out_dim, in_dim))
}
void ref_rms(size_t g0, const float *x, const float *w, float *y, int rows, int width,
             float eps, int affine) {
    RANGE1(g0, refcl::rms(x, w, y, rows, width, eps, affine))
}
void ref_rope(size_t g0, const float *x, const float *freq, const float *pos, float *y,
              int rows, int heads, int dim, int split_half) {
    RANGE1(g0, refcl::rope(x, freq, pos, y, rows, heads, dim, split_half))
}
void ref_swiglu(size_t g0, const float *g, const float *u, float *y, int n) {
    RANGE1(g0, refcl::swiglu(g, u, y, n))
}
void ref_axpy(size_t g0, const float *x, const float *yv, float *z, int n, float scale) {
    RANGE1(g0, refcl::axpy(x, yv, z, n, scale))
}
void ref_scores(size_t g0, size_t g1, const float *q, const float *k, const float *extra_k,
                float *s, int heads, int kv_heads, int dim, int capacity, int start,
                int length, int extra_length) {
    RANGE2(g0, g1, refcl::scores(q, k, extra_k, s, heads, kv_heads, dim, capacity, start,
                                 length, extra_length))
}
void ref_softmax(size_t g0, const float *x, float *y, int rows, int width) {
    RANGE1(g0, refcl::softmax(x, y, rows, width))
}
void ref_latent_mask(size_t g0, size_t g1, float *scores, const float *positions, int heads,
                     int length, int memory, int earliest) {
    RANGE2(g0, g1, refcl::latent_mask(scores, positions, heads, length, memory, earliest))
}
void ref_mix(size_t g0, const float *p, const float *v, const float *extra_v, float *y,
             int heads, int kv_heads, int dim, int capacity, int start, int length,
             int extra_length) {
    RANGE1(g0, refcl::mix(p, v, extra_v, y, heads, kv_heads, dim, capacity, start, length,
                          extra_length))
}
void ref_pool_scores(size_t g0, size_t g1, const float *u, const float *q, float *s,
                     int tokens, int slots, int width) {
    RANGE2(g0, g1, refcl::pool_scores(u, q, s, tokens, slots, width))
}
void ref_pool_mix(size_t g0, size_t g1, const float *u, const float *p, float *z,
                  float *anchors, int tokens, int slots, int width, int start_position) {
    RANGE2(g0, g1, refcl::pool_mix(u, p, z, anchors, tokens, slots, width, start_position))
}
void ref_merge_rows(size_t g0, const float *x, float *y, int width, float a, float b) {
    RANGE1(g0, refcl::merge_rows(x, y, width, a, b))
}
void ref_block_means(size_t g0, size_t g1, const float *x, float *y, int length, int width,
                     int block) {
    RANGE2(g0, g1, refcl::block_means(x, y, length, width, block))
}

}  // extern "C"
