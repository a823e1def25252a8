// Operations on a model's resident tensors, in their stored dtype.
//
// The decode engine (engine_kernel.cu) covers the grouped-query families.  For
// the others (flashnano-1.6 chunk relays, FlashLighting latent attention,
// Heavy Medium sparse attention + MoE) the token step runs on the host over
// the op kernels (ops.cu), exactly as the reference's model.py drives its
// OpenCL kernels -- but the weights stay resident in HBM in the checkpoint's
// dtype instead of being widened on the host and re-uploaded through an LRU.
// These entry points give that host loop what the reference's WeightCache
// gave it (weights.py:258-297): a projection against a named tensor, and the
// widened contents of small tensors.
//
// mr_model_linear follows the reference's linear kernel (kernels.cl:5-17)
// operation for operation: per output, four running sums over j mod 4 in
// increasing j, combined as ((s0 + s1) + s2) + s3, then the tail elements in
// order, every product and sum rounded separately (FP_CONTRACT OFF).  Stored
// BF16/F16 weights widen to float32 exactly, so the result equals the
// reference's linear over its host-widened weights bit for bit.
#include <algorithm>

#include "common.cuh"

namespace mr {

// engine.cu
int model_tensor(mr_model *m, const char *name, const void **ptr, int *dtype, int64_t *rows, int64_t *cols);
int model_stream(mr_model *m, cudaStream_t *stream, int *device);

namespace {

constexpr int kOutTile = 128;  // outputs per block (one thread each)
constexpr int kKTile = 32;     // input elements staged per step (a multiple of 4: keeps j mod 4)

template <int DT>
__device__ __forceinline__ float widen(const void *base, size_t i) {
    if (DT == MR_DTYPE_F32) return static_cast<const float *>(base)[i];
    const uint16_t bits = static_cast<const uint16_t *>(base)[i];
    return DT == MR_DTYPE_BF16 ? widen_bf16(bits) : widen_f16(bits);
}

// y[r, o] = x[r, :] . W[o, :]; grid (ceil(out / kOutTile), rows).
template <int DT>
__global__ void __launch_bounds__(kOutTile) k_linear_stored(const float *x, const void *w, float *y, int out_dim,
                                                            int in_dim) {
    __shared__ float wt[kOutTile][kKTile + 1];
    __shared__ float xt[kKTile];
    const int o0 = blockIdx.x * kOutTile, r = blockIdx.y, t = threadIdx.x, o = o0 + t;
    const float *xr = x + static_cast<size_t>(r) * in_dim;
    const int body = in_dim - in_dim % 4;  // the four-lane part; the rest is the serial tail
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < body; k0 += kKTile) {
        const int kn = min(kKTile, body - k0);
        for (int idx = t; idx < kOutTile * kKTile; idx += kOutTile) {
            const int row = idx / kKTile, col = idx % kKTile;
            wt[row][col] = (o0 + row < out_dim && col < kn)
                               ? widen<DT>(w, static_cast<size_t>(o0 + row) * in_dim + k0 + col)
                               : 0.f;
        }
        if (t < kKTile) xt[t] = t < kn ? xr[k0 + t] : 0.f;
        __syncthreads();
        for (int jj = 0; jj < kn; ++jj) s[jj & 3] = __fadd_rn(s[jj & 3], __fmul_rn(xt[jj], wt[t][jj]));
        __syncthreads();
    }
    if (o >= out_dim) return;
    float v = __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[1]), s[2]), s[3]);
    for (int j = body; j < in_dim; ++j) v = __fadd_rn(v, __fmul_rn(xr[j], widen<DT>(w, static_cast<size_t>(o) * in_dim + j)));
    y[static_cast<size_t>(r) * out_dim + o] = v;
}

template <int DT>
__global__ void k_widen(const void *src, float *dst, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        dst[i] = widen<DT>(src, i);
}

int widen_to(const void *src, int dtype, float *dst, size_t n, cudaStream_t stream) {
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 4096));
    switch (dtype) {
        case MR_DTYPE_BF16: k_widen<MR_DTYPE_BF16><<<blocks, 256, 0, stream>>>(src, dst, n); break;
        case MR_DTYPE_F16: k_widen<MR_DTYPE_F16><<<blocks, 256, 0, stream>>>(src, dst, n); break;
        default: k_widen<MR_DTYPE_F32><<<blocks, 256, 0, stream>>>(src, dst, n); break;
    }
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

}  // namespace
}  // namespace mr

extern "C" {

int mr_model_linear(mr_model *m, const char *name, const mr_buffer *x, int rows, mr_buffer *y) {
    MR_REQUIRE(m && name && x && y, "NULL argument");
    const void *w = nullptr;
    int dtype = 0, device = 0;
    int64_t out_dim = 0, in_dim = 0;
    cudaStream_t stream = nullptr;
    int rc = mr::model_tensor(m, name, &w, &dtype, &out_dim, &in_dim);
    if (!rc) rc = mr::model_stream(m, &stream, &device);
    if (rc) return rc;
    MR_REQUIRE(rows > 0, "rows must be positive");
    MR_REQUIRE(x->count >= static_cast<size_t>(rows) * in_dim, "x holds %zu floats, need %lld", x->count,
               static_cast<long long>(rows * in_dim));
    MR_REQUIRE(y->count >= static_cast<size_t>(rows) * out_dim, "y holds %zu floats, need %lld", y->count,
               static_cast<long long>(rows * out_dim));
    MR_REQUIRE(rows <= 65535, "rows %d above the launch limit", rows);
    MR_CUDA_TRY(cudaSetDevice(device));
    const dim3 grid(static_cast<unsigned>((out_dim + mr::kOutTile - 1) / mr::kOutTile), static_cast<unsigned>(rows));
    const int od = static_cast<int>(out_dim), id = static_cast<int>(in_dim);
    switch (dtype) {
        case MR_DTYPE_BF16: mr::k_linear_stored<MR_DTYPE_BF16><<<grid, mr::kOutTile, 0, stream>>>(x->ptr, w, y->ptr, od, id); break;
        case MR_DTYPE_F16: mr::k_linear_stored<MR_DTYPE_F16><<<grid, mr::kOutTile, 0, stream>>>(x->ptr, w, y->ptr, od, id); break;
        default: mr::k_linear_stored<MR_DTYPE_F32><<<grid, mr::kOutTile, 0, stream>>>(x->ptr, w, y->ptr, od, id); break;
    }
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

int mr_model_tensor_rows(mr_model *m, const char *name, int64_t row0, int64_t nrows, mr_buffer *out) {
    MR_REQUIRE(m && name && out, "NULL argument");
    const void *w = nullptr;
    int dtype = 0, device = 0;
    int64_t rows = 0, cols = 0;
    cudaStream_t stream = nullptr;
    int rc = mr::model_tensor(m, name, &w, &dtype, &rows, &cols);
    if (!rc) rc = mr::model_stream(m, &stream, &device);
    if (rc) return rc;
    MR_REQUIRE(row0 >= 0 && nrows > 0 && row0 + nrows <= rows, "rows [%lld, %lld) outside %s [%lld, %lld]",
               static_cast<long long>(row0), static_cast<long long>(row0 + nrows), name,
               static_cast<long long>(rows), static_cast<long long>(cols));
    const size_t n = static_cast<size_t>(nrows * cols);
    MR_REQUIRE(out->count >= n, "out holds %zu floats, need %zu", out->count, n);
    MR_CUDA_TRY(cudaSetDevice(device));
    const size_t esz = dtype == MR_DTYPE_F32 ? 4 : 2;
    return mr::widen_to(static_cast<const char *>(w) + static_cast<size_t>(row0 * cols) * esz, dtype, out->ptr, n,
                        stream);
}

int mr_model_tensor_download(mr_model *m, const char *name, float *host, size_t count) {
    MR_REQUIRE(m && name && host, "NULL argument");
    const void *w = nullptr;
    int dtype = 0, device = 0;
    int64_t rows = 0, cols = 0;
    cudaStream_t stream = nullptr;
    int rc = mr::model_tensor(m, name, &w, &dtype, &rows, &cols);
    if (!rc) rc = mr::model_stream(m, &stream, &device);
    if (rc) return rc;
    const size_t n = static_cast<size_t>(rows * cols);
    MR_REQUIRE(count == n, "%s has %zu elements, host buffer %zu", name, n, count);
    MR_CUDA_TRY(cudaSetDevice(device));
    float *tmp = nullptr;
    MR_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void **>(&tmp), n * sizeof(float), stream));
    rc = mr::widen_to(w, dtype, tmp, n, stream);
    cudaError_t err = rc ? cudaSuccess : cudaMemcpyAsync(host, tmp, n * sizeof(float), cudaMemcpyDeviceToHost, stream);
    cudaFreeAsync(tmp, stream);
    if (rc) return rc;
    if (err != cudaSuccess) return mr::cuda_error(err, "tensor download");
    MR_CUDA_TRY(cudaStreamSynchronize(stream));
    return MR_OK;
}

}  // extern "C"
