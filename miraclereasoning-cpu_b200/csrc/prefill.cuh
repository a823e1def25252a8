// Batched prompt processing (prefill) for the grouped-query families:
// the reference's token loop (model.py:295-312) applied to a chunk of T
// prompt tokens at once.  Projections are GEMMs on the tensor cores over BF16
// weights with the FP32 activations split into three BF16 parts
// (x = x0 + x1 + x2, exact to 2^-24 relative), so every product is exact and
// only the FP32 accumulation order differs from the reference's linear
// kernel; attention runs causally over the ring's older keys plus the chunk's
// own, in FP32.
#pragma once

#include <vector>

#include <cuda_bf16.h>

#include "common.cuh"

namespace mr {

struct PrefillLayer {
    const void *a_norm, *f_norm, *q_norm, *k_norm;  // gains (q_norm / k_norm: NULL without q/k norm)
    int a_norm_dt, f_norm_dt, qk_norm_dt;
    const void *q, *k, *v, *o, *gate, *up, *down;    // BF16 matrices [out, in]
    float *k_cache, *v_cache;                        // [kv_heads][capacity][head_dim]
    int capacity, kv_heads;
    // FlashLighting (no memory slots): q | latent and gate | up from a_norm(x),
    // k | v (BF16 [kv, latent]) from latent_norm(latent), residual scales
    // residual_scale * attention_gate and residual_scale * ffn_gate
    const void *latent, *latent_norm;
    int latent_norm_dt;
    float o_scale, down_scale;
};

struct PrefillModel {
    cudaStream_t stream;
    int hidden, heads, head_dim, ffn, vocab, kv_max;
    float eps, residual_scale;
    int qk_norm, split_half;
    int lighting, latent_dim;  // FlashLighting layers (PrefillLayer's latent path)
    const void *embed;  // [vocab, hidden] stored dtype
    int embed_dt;
    const void *final_norm;
    int final_norm_dt;
    const void *head;   // BF16 [vocab, hidden] (the embedding when tied)
    const float *inv_freq;  // [head_dim / 2] on the device
    std::vector<PrefillLayer> layers;
};

// Device workspace for chunks of up to `tokens` tokens.
struct PrefillWork {
    int tokens = 0;
    bool all_logits = false;
    float *x = nullptr;        // [T][hidden] residual stream
    uint16_t *planes = nullptr;  // [3][T][kmax] BF16 parts of a GEMM input
    int kmax = 0;
    float *qkv = nullptr;      // [T][q + 2 kv_max]
    float *qh = nullptr;       // [T][heads * d] normalised, rotated queries
    float *kc = nullptr, *vc = nullptr;  // [T][kv_max * d] the chunk's keys / values
    float *gu = nullptr;       // [T][2 ffn]: gate row | up row
    float *logits = nullptr;   // [T or 1][vocab]
    int *err = nullptr;        // a bounded wait of the tcgen05 GEMM gave up
    bool tcgen05 = true;       // GEMMs on tcgen05 (else mma.sync, kept as the comparison baseline)
};

// Allocates (or grows) the workspace on the model's stream.
int prefill_reserve(const PrefillModel &pm, PrefillWork &w, int tokens, bool all_logits);
void prefill_release(PrefillWork &w);

// Reads back the GEMMs' wait status (synchronises the stream).
int prefill_status(const PrefillModel &pm, PrefillWork &w);

// Runs T tokens (device ids) at positions p0 .. p0 + T - 1 through every
// layer, appending their keys and values to the rings, and writes the logits
// of every token (all_logits) or of the last one into w.logits.
int prefill_chunk(const PrefillModel &pm, PrefillWork &w, const int *d_ids, int T, int p0, bool all_logits);

// ---- building blocks shared with Heavy Medium's batched prompt (heavy_prefill.cuh) ----

// One BF16 weight matrix [n][K] (row-major) whose products land in output
// columns col0 .. col0 + n - 1.
struct BatchSeg {
    const void *w;
    int n, col0;
};

// Y[m][col0 + j] = sum_k X[m][k] W[j][k] (resid: Y = Y + scale * that) for M
// rows of X given as BF16x3 planes ([3][rows][lda], plane_stride elements
// apart), up to 3 segments, on tcgen05 (*err: a bounded wait gave up).
int batch_gemm(cudaStream_t stream, int *err, const uint16_t *planes, size_t plane_stride, int lda, int M, int K,
               const BatchSeg *segs, int nseg, float *y, int ldy, bool resid, float scale);

// Grouped form: grid row y < *tile_count takes tiles[y] = {group, row0, row_end}:
// X rows [row0, row0 + 128) against group's weights (maps[group * nseg + s],
// encoded by batch_weight_map), output rows below row_end only.  `segs`
// gives each segment's n and col0 (its w is not read); max_tiles bounds the grid.
int batch_gemm_grouped(cudaStream_t stream, int *err, const uint16_t *planes, size_t plane_stride, int lda, int rows,
                       int K, const void *maps, const BatchSeg *segs, int nseg, const int *tiles,
                       const int *tile_count, int max_tiles, float *y, int ldy);
constexpr int kBatchTileRows = 128;  // X rows per tile of batch_gemm_grouped
constexpr size_t kBatchMapBytes = 128;  // one encoded weight map

// Encodes the tensor map batch_gemm_grouped reads for a BF16 [n][K] matrix
// into `map` (kBatchMapBytes, host memory; copy it to the device array).
int batch_weight_map(void *map, const void *w, int n, int K);

// planes[i] = split(RMSNorm(x[row0 + i]) * gain) for `rows` rows of width h
// (gain NULL: 1), kernels.cl:19-28.
int batch_rms_planes(cudaStream_t stream, const float *x, int row0, int rows, int h, int ldx, const void *gain,
                     int gain_dt, float eps, uint16_t *planes, size_t plane_stride, int ld);

// Shared-memory opt-ins of the GEMM kernels (once per device).
int batch_setup();

#ifdef __CUDACC__
// x = p0 + p1 + p2 in BF16 parts (each residual is exact in FP32), the form
// every batched GEMM input takes.
__device__ __forceinline__ uint16_t bf16_bits(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ float bf16_value(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ void put_planes(uint16_t *planes, size_t plane_stride, size_t idx, float v) {
    const uint16_t a = bf16_bits(v);
    const float r1 = __fsub_rn(v, bf16_value(a));
    const uint16_t b = bf16_bits(r1);
    const float r2 = __fsub_rn(r1, bf16_value(b));
    planes[idx] = a;
    planes[plane_stride + idx] = b;
    planes[2 * plane_stride + idx] = bf16_bits(r2);
}
#endif

}  // namespace mr
