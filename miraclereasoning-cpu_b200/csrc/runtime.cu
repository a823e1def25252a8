// Errors, devices, contexts and float32 buffers of libmiracle_cuda.so.
//
// Buffers replace the reference's clCreateBuffer-per-op tensors
// (miracle_reasoning/opencl.py:178-217): sizes/offsets in float elements,
// blocking upload/download, bounds-checked device-to-device copies.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace mr {

static thread_local char g_error[1024] = "";

int set_error(int code, const char *fmt, ...) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, args);
    va_end(args);
    return code;
}

int cuda_error(cudaError_t err, const char *what) {
    return set_error(err == cudaErrorMemoryAllocation ? MR_ERR_NOMEM : MR_ERR_CUDA, "%s failed: %s (%s)",
                     what, cudaGetErrorString(err), cudaGetErrorName(err));
}

}  // namespace mr

extern "C" {

const char *mr_last_error(void) { return mr::g_error; }
int mr_abi_version(void) { return MR_ABI_VERSION; }

int mr_device_count(int *count) {
    MR_REQUIRE(count, "count is NULL");
    int n = 0;
    cudaError_t err = cudaGetDeviceCount(&n);
    if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *count = 0;
        return MR_OK;
    }
    MR_CUDA_TRY(err);
    *count = n;
    return MR_OK;
}

int mr_device_query(int ordinal, mr_device_info *info) {
    MR_REQUIRE(info, "info is NULL");
    cudaDeviceProp prop;
    MR_CUDA_TRY(cudaGetDeviceProperties(&prop, ordinal));
    memset(info, 0, sizeof(*info));
    info->ordinal = ordinal;
    info->sm_count = prop.multiProcessorCount;
    info->cc_major = prop.major;
    info->cc_minor = prop.minor;
    info->memory_bytes = prop.totalGlobalMem;
    info->max_allocation_bytes = prop.totalGlobalMem;
    snprintf(info->name, sizeof(info->name), "%s", prop.name);
    return MR_OK;
}

int mr_context_create(int device_ordinal, mr_context **out) {
    MR_REQUIRE(out, "out is NULL");
    int count = 0;
    int rc = mr_device_count(&count);
    if (rc) return rc;
    MR_REQUIRE(device_ordinal >= 0 && device_ordinal < count,
               "no CUDA device %d (found %d); this engine has no CPU fallback", device_ordinal, count);
    cudaDeviceProp prop;
    MR_CUDA_TRY(cudaGetDeviceProperties(&prop, device_ordinal));
    if (prop.major < 10)
        return mr::set_error(MR_ERR_ARGUMENT, "device %d (%s, sm_%d%d) is not a Blackwell sm_100 part",
                             device_ordinal, prop.name, prop.major, prop.minor);
    MR_CUDA_TRY(cudaSetDevice(device_ordinal));
    auto *ctx = new mr_context();
    ctx->device = device_ordinal;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->max_allocation = prop.totalGlobalMem;
    cudaError_t err = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
        delete ctx;
        return mr::cuda_error(err, "cudaStreamCreate");
    }
    *out = ctx;
    return MR_OK;
}

int mr_context_destroy(mr_context *ctx) {
    if (ctx) mr::context_release(ctx);
    return MR_OK;
}

int mr_context_finish(mr_context *ctx) {
    MR_REQUIRE(ctx, "ctx is NULL");
    MR_CUDA_TRY(cudaSetDevice(ctx->device));
    MR_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return MR_OK;
}

int mr_buffer_alloc(mr_context *ctx, size_t count, mr_buffer **out) {
    MR_REQUIRE(ctx && out, "NULL argument");
    MR_REQUIRE(count > 0, "invalid buffer size 0");
    MR_REQUIRE(count <= ctx->max_allocation / 4, "buffer of %zu floats exceeds device memory", count);
    MR_CUDA_TRY(cudaSetDevice(ctx->device));
    float *ptr = nullptr;
    MR_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void **>(&ptr), count * sizeof(float), ctx->stream));
    auto *buf = new mr_buffer();
    mr::context_retain(ctx);
    buf->ctx = ctx;
    buf->ptr = ptr;
    buf->count = count;
    *out = buf;
    return MR_OK;
}

int mr_buffer_free(mr_buffer *buf) {
    if (!buf) return MR_OK;
    cudaSetDevice(buf->ctx->device);
    cudaFreeAsync(buf->ptr, buf->ctx->stream);
    mr::context_release(buf->ctx);
    delete buf;
    return MR_OK;
}

int mr_buffer_count(const mr_buffer *buf, size_t *count) {
    MR_REQUIRE(buf && count, "NULL argument");
    *count = buf->count;
    return MR_OK;
}

int mr_buffer_upload(mr_buffer *buf, size_t offset, const float *host, size_t count) {
    MR_REQUIRE(buf && (host || !count), "NULL argument");
    MR_REQUIRE(offset <= buf->count && count <= buf->count - offset, "upload is out of bounds");
    if (!count) return MR_OK;
    MR_CUDA_TRY(cudaSetDevice(buf->ctx->device));
    MR_CUDA_TRY(cudaMemcpyAsync(buf->ptr + offset, host, count * sizeof(float), cudaMemcpyHostToDevice,
                                buf->ctx->stream));
    MR_CUDA_TRY(cudaStreamSynchronize(buf->ctx->stream));
    return MR_OK;
}

int mr_buffer_download(const mr_buffer *buf, size_t offset, float *host, size_t count) {
    MR_REQUIRE(buf && (host || !count), "NULL argument");
    MR_REQUIRE(offset <= buf->count && count <= buf->count - offset, "read is out of bounds");
    if (!count) return MR_OK;
    MR_CUDA_TRY(cudaSetDevice(buf->ctx->device));
    MR_CUDA_TRY(cudaMemcpyAsync(host, buf->ptr + offset, count * sizeof(float), cudaMemcpyDeviceToHost,
                                buf->ctx->stream));
    MR_CUDA_TRY(cudaStreamSynchronize(buf->ctx->stream));
    return MR_OK;
}

int mr_buffer_copy(const mr_buffer *src, mr_buffer *dst, size_t src_offset, size_t dst_offset,
                   size_t count) {
    MR_REQUIRE(src && dst, "NULL buffer");
    MR_REQUIRE(src->ctx == dst->ctx, "Tensors belong to different CUDA contexts");
    MR_REQUIRE(src_offset <= src->count && count <= src->count - src_offset && dst_offset <= dst->count &&
                   count <= dst->count - dst_offset,
               "tensor copy is out of bounds");
    if (!count) return MR_OK;
    MR_CUDA_TRY(cudaSetDevice(src->ctx->device));
    MR_CUDA_TRY(cudaMemcpyAsync(dst->ptr + dst_offset, src->ptr + src_offset, count * sizeof(float),
                                cudaMemcpyDeviceToDevice, src->ctx->stream));
    return MR_OK;
}

}  // extern "C"
