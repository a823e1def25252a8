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

}  // namespace mr
