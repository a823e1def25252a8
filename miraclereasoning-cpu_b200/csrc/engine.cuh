// Whole-model decode engine: data structures shared by the host planner
// (engine.cu) and the persistent decode kernel (engine_kernel.cu).
//
// One decode step of the reference token loop (miracle_reasoning/model.py:
// 257-285 and the head at 307) is compiled on the host into a fixed list of
// PHASES.  A phase is a unit of work that needs the complete results of the
// previous phase (a GEMV needs the whole input vector; attention needs all of
// this token's q/k/v).  The decode kernel is launched cooperatively with one
// CTA per SM and runs every phase of a step, separated by grid-wide barriers;
// inside a phase each CTA takes its share of the work.  Before a phase starts
// computing, its CTA issues L2 bulk prefetches for its share of the NEXT
// weight-streaming phase, so HBM keeps streaming through the barriers.
#pragma once

#include "common.cuh"

namespace mr {

constexpr int kEngineThreads = 512;  // 16 warps per CTA, one CTA per SM
constexpr int kEngineWarps = kEngineThreads / 32;
constexpr int kMaxSegments = 3;
constexpr int kMaxInput = 16384;     // floats of one GEMV input vector held in shared memory
constexpr int kRowBatch = 256;       // local rows per GEMV epilogue batch
constexpr int kMergeSlots = 2048;    // (query head, chunk) softmax weights staged for a merge

enum PhaseKind : int {
    PH_GEMV = 1,        // y = W x for up to 3 weight segments, then an epilogue
    PH_ATTN_GQA = 2,    // q/k norm + RoPE + ring append + attention (+ relay rows)
    PH_STEP_END = 3,    // argmax bookkeeping, position advance
};

enum Epilogue : int {
    EPI_STORE = 0,      // out_s[r] = y_s[r] for every segment s
    EPI_RESIDUAL = 1,   // x[r] = x[r] + scale * y_0[r]              (kernels.cl:52-56)
    EPI_SWIGLU = 2,     // out[r] = (g/(1+exp(-g))) * u, g=y_0, u=y_1 (kernels.cl:46-50)
    EPI_LOGITS = 3,     // logits[r] = y_0[r]; running argmax
};

enum InputKind : int {
    IN_VECTOR = 0,      // a float vector in global memory
    IN_EMBED_ROW = 1,   // row `token` of the embedding, widened
};

struct Segment {
    const void *w;      // [rows, cols] row-major, stored dtype
    int dtype;
    int rows, cols;
    float *out;         // EPI_STORE destination (rows floats)
};

struct GemvPhase {
    int input_kind;
    const float *in;            // IN_VECTOR source (cols floats)
    const void *embed;          // IN_EMBED_ROW source [vocab, cols]
    int embed_dtype;
    float *embed_copy;          // when set, CTA 0 also stores the widened row here
    int norm;                   // apply RMSNorm to the input
    const void *norm_gain;      // NULL -> non-affine
    int norm_gain_dtype;
    float norm_eps;
    int nseg;
    Segment seg[kMaxSegments];
    int epilogue;
    float scale;                // EPI_RESIDUAL scale
    float *x;                   // EPI_RESIDUAL vector
    float *out;                 // EPI_SWIGLU / EPI_LOGITS destination
};

struct AttnPhase {
    const float *q_raw, *k_raw, *v_raw;
    int qk_norm;                    // per-head RMSNorm of q and k before RoPE
    const void *q_gain, *k_gain;    // its gains (NULL: non-affine)
    int gain_dtype;
    float norm_eps;
    int heads, kv_heads, dim;
    int split_half;
    const float *inv_freq;
    float *k_cache, *v_cache;       // [kv_heads][capacity][dim]
    int capacity;
    const float *relay_k, *relay_v; // [kv_heads][relay_capacity][dim] (flashnano-1.6) or NULL
    const int *relay_count;
    int relay_capacity;
    float *partial;                 // [heads][max_chunks][dim + 2]
    unsigned int *arrivals;         // [kv_heads]
    int max_chunks;
    float *out;                     // [heads * dim]
};

struct Phase {
    int kind;
    int layer;                      // -1: the output head (skipped when no logits are needed)
    GemvPhase gemv;
    AttnPhase attn;
};

// Device-resident state of the running sequence, advanced by the decode
// kernel itself (CTA 0, after the step's final barrier) so that steps can be
// queued back to back without the host.
struct StepState {
    unsigned long long barrier;       // monotonic grid-barrier counter
    unsigned long long barrier_base;  // its value when the current launch began
    unsigned long long best;          // packed argmax of the current step
    int position;                     // position of the token being processed
    int token;                        // next token when it is not fed (greedy)
    int gen_count;                    // tokens generated so far
    int stopped;                      // generation finished: further launches do nothing
    int nonfinite;                    // a non-finite logit was produced
    int last_argmax;
    int error;                        // nonzero: 1000 + phase = a bounded wait gave up, 3 = context full, 4 = bad token
};

// Per-launch control, passed by value.
struct StepControl {
    const int *feed;                  // tokens of the current prefill
    int feed_base, feed_len;          // feed[i] is the token at position feed_base + i
    int return_all;                   // logits for every fed token (else last only)
    int logits_rows;                  // logits ring: row (position - feed_base) % logits_rows
    int gen_max, eos;                 // device greedy generation (gen_max 0 = off)
    int *gen_out;
    int context_length;
    int vocab_size;                   // tokens outside [0, vocab) stop the step with error 4
    // Optional phase trace (globaltimer ns): [0] = launch start (CTA 0); then per
    // executed phase k, slots 1 + k*(grid+1) + b = CTA b done computing, and
    // slot 1 + k*(grid+1) + grid = CTA 0 leaving the barrier.  NULL = off.
    unsigned long long *trace;
};

}  // namespace mr
