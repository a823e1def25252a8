// Heavy Medium 2.0 on the device (heavy.cu): the token step of
// miracle_reasoning/model.py:192-285 as kernel launches, with the block top-k
// and the expert routing taken on the GPU.
#pragma once

#include "common.cuh"

namespace mr {

struct HeavyEngine;

// Reads the model's resident tensors (the model must be finalized) and
// allocates the work buffers and one key/value ring per (layer, inner loop).
// With ranks > 1 (expert parallel) every rank runs the attention, router and
// head itself and the experts e with e % ranks == rank, exchanging expert rows
// through an arena that every rank maps (heavy_arena / heavy_connect).
int heavy_create(mr_model *m, const mr_model_config &c, cudaStream_t stream, const float *inv_freq_host, int rank,
                 int ranks, HeavyEngine **out);
void heavy_arena(const HeavyEngine *e, char **arena, size_t *bytes);
void heavy_connect(HeavyEngine *e, char *const *peers);
// Reads the wait status of the expert-parallel exchange (synchronous).
int heavy_status(const HeavyEngine *e);
void heavy_destroy(HeavyEngine *e);
// A new sequence: zeroes the device counters of the fused kernels and the error word.
int heavy_reset(HeavyEngine *e);
// How long the kernels' bounded waits last (default 2 s).
int heavy_set_wait_limit(HeavyEngine *e, unsigned long long nanoseconds);
// Fault injection for tests: while on, the attention units do not count their
// key / value rows, so the units that need the new row wait until their limit.
int heavy_inject_fault(HeavyEngine *e, bool on);

// float32 log1p(d) for distances d = 0 .. context-1, as the host computes them
// (the reference applies NumPy's float32 log1p, model.py:221-222).
int heavy_set_log1p(HeavyEngine *e, const float *values, int n);

// Queues one token at `position` on the engine's stream; the logits (vocab
// floats) are then at heavy_logits(e).
int heavy_token(HeavyEngine *e, int token, int position);
const float *heavy_logits(const HeavyEngine *e);

// heavy_token with a %globaltimer stamp before the step and after every kernel
// (stamps[0] = start, stamps[k] = completion of the step's k-th kernel);
// synchronous.  *count receives the number of stamps written.
int heavy_trace_token(HeavyEngine *e, int token, int position, unsigned long long *stamps, int capacity, int *count);

// The token step with its input token read from heavy_token_slot(e) (device
// sampling writes it there), and that slot.
int heavy_token_from_slot(HeavyEngine *e, int position);
int *heavy_token_slot(HeavyEngine *e);

// Batched prompt (heavy_prefill.cuh): T tokens (host ids) at positions p0 ..
// p0 + T - 1 through every layer at once, GEMMs on tcgen05, leaving the state
// heavy_token continues from; the logits of every token (all_logits) or of the
// last one are then at heavy_prefill_logits(e).  Only for models with
// heavy_batchable (BF16 matrices, one engine).
bool heavy_batchable(const HeavyEngine *e);
int heavy_prefill(HeavyEngine *e, const int *ids, int T, int p0, bool all_logits);
const float *heavy_prefill_logits(const HeavyEngine *e);

// Greedy decode entirely on the device: `steps` tokens from `position`, each
// step's input the previous step's argmax (the first: first_token).
int heavy_greedy_chain(HeavyEngine *e, int first_token, int position, int steps);

// Decisions of the last token (synchronise the stream): kept block ids
// (heads x global_slots, ascending per head, -1 padded) and the experts in
// rank order with their weights (router_top_k_max entries, -1 / 0 padded).
int heavy_last_topk(const HeavyEngine *e, int layer, int loop, int *blocks, int capacity);
int heavy_last_experts(const HeavyEngine *e, int layer, int loop, int *experts, float *weights, int capacity);

}  // namespace mr
