// Whole-model decode engine: data structures shared by the host planner
// (engine.cu) and the persistent decode kernel (engine_kernel.cu).
//
// One decode step of the reference token loop (miracle_reasoning/model.py:
// 257-285 and the head at 307) is compiled on the host into a fixed list of
// PHASES.  A phase is a unit of work that needs the complete results of the
// previous phase (a GEMV needs the whole input vector; attention needs all of
// this token's q/k/v).  The decode kernel is launched cooperatively with one
// CTA per SM and runs every phase of a step, separated by grid-wide barriers;
// inside a phase each CTA takes its share of the work.
//
// Data exchange between phases: every vector one phase hands to the next (the
// residual stream x, q/k/v rows, attention chunk partials, the SwiGLU
// activation) is stored as 64-bit words {float value (low half), tag (high
// half)}, written and read with single-copy-atomic 64-bit accesses.  The tag
// names the launch and the producing phase, so a reader polls its words until
// they carry the expected tag: no grid barrier between phases, one L2 round
// trip from the last write to the reader.  Every phase reads what the phase
// before it wrote (expected tag = tag_base + p - 1).  A buffer is rewritten
// only after every reader of its previous contents has finished, because each
// writer's own inputs depend, through the phase chain, on every such reader
// having produced its output -- which is why a CTA that has no output in a
// phase reads none of its input either.
//
// Weight streaming: every CTA owns a fixed row range of each weight segment.
// A dedicated producer warp walks the CTA's slices of all weight-streaming
// phases of the step, in order, as "pieces" (whole rows of one segment, or a
// norm gain vector) and copies them with TMA bulk copies (cp.async.bulk, one
// "full" mbarrier per piece) into a shared-memory byte ring, as far ahead as
// the ring has room -- across phase boundaries and grid barriers.  The 16
// compute warps consume the pieces in the same order and hand each slot back
// through an "empty" mbarrier.  The compute of a phase reads its weights from
// shared memory, so the only global round trips left on its critical path are
// the phase's input vector and the barrier.
#pragma once

#include "common.cuh"

namespace mr {

// 15 compute warps + 1 producer warp: 16 warps, 4 per SM sub-partition, so
// each thread may hold 128 registers (a 17th warp would cap it at 96).
constexpr int kEngineThreads = 480;  // compute threads per CTA, one CTA per SM
constexpr int kEngineWarps = kEngineThreads / 32;
constexpr int kBlockThreads = kEngineThreads + 32;  // + the weight-stream producer warp
constexpr int kMaxSegments = 3;
constexpr int kRowBatch = 256;       // rows of one piece (and of one direct-load batch)
constexpr int kQueue = 32;           // pieces in flight per CTA (one mbarrier each)
constexpr int kMaxAttnChunks = 64;   // key chunks per KV head (at most grid / KV heads are used)
constexpr int kKeysPerChunk = 64;    // target keys per attention work unit
constexpr int kKeyTile = 64;         // keys per attention tile
constexpr int kSmemLimit = 227 * 1024;
constexpr int kTraceStamps = 6;

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
    EPI_RESIDUAL_KEEP = 4,  // as EPI_RESIDUAL, but only this CTA's shared-memory rows are updated (a
                            // later residual phase of the layer publishes them)
};

enum InputKind : int {
    IN_VECTOR = 0,      // a float vector in global memory
    IN_EMBED_ROW = 1,   // row `token` of the embedding, widened
};

typedef unsigned long long Word;  // exchanged value: float bits | tag << 32

struct Segment {
    const void *w;      // [rows, cols] row-major, stored dtype
    int dtype;
    int rows, cols;
    int rows_per_piece; // rows per bulk piece (bulk phases)
    Word *out;          // EPI_STORE destination (rows words)
    int row_lo, row_n;  // this rank's rows (tensor parallel: a contiguous slice; else all)
};

constexpr int kMaxRanks = 8;  // tensor-parallel ranks (one GPU each)

// Rows [lo, lo + n) of `rows` owned by rank r of `ranks` (contiguous slices).
__host__ __device__ inline void rank_rows(int rows, int r, int ranks, int &lo, int &n) {
    lo = static_cast<int>(static_cast<long long>(rows) * r / ranks);
    n = static_cast<int>(static_cast<long long>(rows) * (r + 1) / ranks) - lo;
}

struct GemvPhase {
    int input_kind;
    const Word *in;             // IN_VECTOR source (cols words)
    const void *embed;          // IN_EMBED_ROW source [vocab, cols]
    int embed_dtype;
    int norm;                   // apply RMSNorm to the input
    const void *norm_gain;      // NULL -> non-affine
    int norm_gain_dtype;
    float norm_eps;
    int gain_piece;             // the gain vector travels through the ring as the phase's first piece
    int nseg;
    Segment seg[kMaxSegments];
    int bulk;                   // weights stream through the shared-memory ring
    int epilogue;
    float scale;                // EPI_RESIDUAL scale
    Word *x;                    // EPI_RESIDUAL: the residual stream (this CTA keeps its rows in shared memory)
    Word *out;                  // EPI_SWIGLU destination
    float *logits;              // EPI_LOGITS destination
    int wdtype;                 // bulk: the segments' common dtype, -1 when they differ
    int xsplit;                 // the input vector is staged split for 16-bit weights (see XView)
    int group_offset;           // bulk: this phase's group tables in StepControl::groups,
    int group_stride;           //   CTA b's g-th at group_offset + b * group_stride + g
    int skip;                   // CTAs 0 .. skip-1 own no rows of the phase (see cta_row_range)
    int in_back;                // the input words carry the tag of the phase this many phases back
    float *save_in;             // or NULL: the raw input row is also stored at row position % save_rows
    int save_rows;              //   (flashnano-1.6 chunk inputs, FlashLighting latents; aux_step.cuh)
};

// Rows [r0, r1) of segment s owned by CTA b of G: the CTA's share of the
// rank's slice of the segment.
__host__ __device__ inline void seg_cta_rows(const Segment &s, int b, int G, int skip, int &r0, int &r1);

struct AttnPhase {
    const Word *q_raw, *k_raw, *v_raw;
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
    Word *partial;                  // [heads][kMaxAttnChunks][dim + 2]: chunks 1.. (acc[dim], max, sum)
    Word *out;                      // [heads * dim] attention output (the o projection's input)
    int kv_lo, kv_n;                // this rank's KV heads (tensor parallel: a contiguous slice; else all)
    int q_back;                     // the q words come from the phase this many phases back (k / v: 1)
};

// The compute warps take a bulk phase's pieces in groups, precomputed on the
// host per (phase, CTA): consecutive pieces (a SwiGLU gate/up pair is never
// split) of at most half the ring of rows, or two thirds in phases that
// stream more than half a ring per CTA (plus, in the first group, the norm
// gain vector), kRowBatch rows and kGroupPieces pieces, awaited together and
// computed in one pass.  Every older piece has been released when a group is
// awaited and pieces are at most a quarter (a sixth) of the ring, so a whole
// group, its gain piece and less than a piece lost to a wrap always fit in
// the ring at once.
constexpr int kGroupPieces = kQueue / 2;

struct GroupPiece {
    int seg;     // segment, -1: the phase's norm gain vector
    int row0;    // first output row
    int n;       // rows
    int vbase;   // index of its first row among the group's rows
};
struct alignas(16) GroupTable {
    GroupPiece p[kGroupPieces];
    int count;   // pieces
    int rows;    // dot products
    int more;    // another group of the phase follows
    int pad;
};
static_assert(sizeof(GroupTable) % 16 == 0, "GroupTable travels in 16-byte granules");

// One bulk copy of a CTA's weight stream, precomputed on the host: the CTA's
// pieces of every weight-streaming phase of a step, in consumption order.
// 16 bytes, so the producer fetches each with one vector load.
struct alignas(16) PieceDesc {
    const void *src;    // global source (16-byte aligned)
    uint32_t bytes;     // multiple of 16
    int phase;          // index in the phase list
};
static_assert(sizeof(PieceDesc) == 16, "PieceDesc is one 16-byte load");

// 16-byte aligned and sized: the kernel prefetches the next phase into shared
// memory with 16-byte asynchronous copies.
struct alignas(16) Phase {
    int kind;
    int layer;                      // -1: the output head (skipped when no logits are needed)
    int next_groups;                // the next phase's group tables (its gemv.group_offset) or -1
    int next_group_stride;          //   and its gemv.group_stride: prefetched with its descriptor
    GemvPhase gemv;
    AttnPhase attn;
};
static_assert(sizeof(Phase) % 16 == 0, "Phase must be a whole number of 16-byte granules");

// Attention work split: chunks of keys per KV head (same formula in the
// attention phase and in the merge that consumes its partials).
// Rows [r0, r1) of a `rows`-row matrix owned by CTA b of G when the first
// `skip` CTAs own none (they run the attention units, which would otherwise
// make them the last to finish the phases next to attention).
__host__ __device__ inline void cta_row_range(int rows, int b, int G, int skip, int &r0, int &r1) {
    if (b < skip) {
        r0 = r1 = 0;
        return;
    }
    r0 = static_cast<int>(static_cast<long long>(rows) * (b - skip) / (G - skip));
    r1 = static_cast<int>(static_cast<long long>(rows) * (b + 1 - skip) / (G - skip));
}

__host__ __device__ inline void seg_cta_rows(const Segment &s, int b, int G, int skip, int &r0, int &r1) {
    cta_row_range(s.row_n, b, G, skip, r0, r1);
    r0 += s.row_lo;
    r1 += s.row_lo;
}

__host__ __device__ inline int attn_chunks(int total_keys, int kv_heads, int grid) {
    int chunks = kv_heads > 0 ? grid / kv_heads : 1;  // a rank can hold no KV head of a layer
    const int by_keys = (total_keys + kKeysPerChunk - 1) / kKeysPerChunk;
    if (by_keys < chunks) chunks = by_keys;
    if (kMaxAttnChunks < chunks) chunks = kMaxAttnChunks;
    return chunks < 1 ? 1 : chunks;
}

// Shared-memory scratch carve-up (float offsets) of the attention phase for
// one KV group.  Every array starts on a 16-byte boundary; key rows are
// padded to dim + 4 floats so that float4 reads of 8 consecutive keys hit 32
// distinct banks.  After the chunk's last tile the key/value region (`tiles`
// floats from kt) takes the chunk records that merge_slice gathers.
struct AttnLayout {
    int q, knew, vnew, kt, vt, tiles, p, acc, m, l, wm, total;
    int kstride, vstride;
};
__host__ __device__ inline int round4(int x) { return (x + 3) & ~3; }
__host__ __device__ inline AttnLayout attn_layout(int group_heads, int dim) {
    AttnLayout L;
    L.kstride = round4(dim) + 4;
    L.vstride = round4(dim);
    int o = 0;
    L.q = o;    o += round4(group_heads * dim);   // [gq][dim]
    L.knew = o; o += round4(dim);                 // this token's key
    L.vnew = o; o += round4(dim);                 // this token's value
    L.kt = o;                                     // key tile
    L.vt = o + kKeyTile * L.kstride;              // value tile
    int tiles = kKeyTile * (L.kstride + L.vstride);
    const int records = group_heads * dim + kMaxAttnChunks + 3 * group_heads * kMaxAttnChunks;
    if (tiles < records) tiles = records;
    L.tiles = round4(tiles);
    o += L.tiles;
    L.p = o;    o += round4(group_heads * kKeyTile);
    L.acc = o;  o += round4(group_heads * dim);
    L.m = o;    o += round4(2 * group_heads);   // running max, two buffers (tile parity)
    L.l = o;    o += round4(2 * group_heads);   // running sum, two buffers
    L.wm = o;   o += round4(4 * group_heads);   // per-warp max, then sum, of the current tile
    L.total = o;
    return L;
}

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
    int error;                        // 1000 + phase: a bounded wait gave up; 3: context full; 4: bad token
    unsigned long long wait_limit_ns; // a bounded wait gives up after this long (0: 2 s); survives reset
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
    unsigned int tag_base;            // exchange tags of this launch: tag_base + producing phase
    int scratch_floats;               // shared-memory scratch: GEMV input vector, then the attention region
    int attn_base;                    // float offset of the attention region (16-byte aligned)
    const float *inv_freq;            // RoPE inverse frequencies [rope_pairs], shared by every layer
    int rope_pairs;
    const void *embed;                // embedding [vocab, hidden]: this CTA's rows of the residual stream
    int embed_dtype, hidden;          //   start as the token's embedding
    int xres_skip;                    // CTAs owning no residual rows (cta_row_range)
    int xres_lo, xres_n;              // this rank's rows of the residual stream
    // Tensor parallel: every exchange word (and logit) goes to the same offset
    // of every rank's exchange arena; readers poll their own.
    int ranks;                        // 1: single GPU
    char *arena;                      // this rank's arena (the base of every exchange buffer)
    char *peers[kMaxRanks];           // every rank's arena, mapped here (peers[rank] == arena)
    Word *best_slots;                 // [kMaxRanks][4] step-end argmax exchange (this rank's arena)
    int rank;
    int ring_bytes;                   // shared-memory weight ring
    const PieceDesc *pieces;          // [grid][piece_stride] weight stream of each CTA
    const GroupTable *groups;         // piece groups of every (bulk phase, CTA)
    const int *piece_count;           // [grid]
    int piece_stride;
    // Optional phase trace (globaltimer ns): [0] = launch start (CTA 0); then per
    // executed phase k a record of grid*kTraceStamps + 1 slots: CTA b's slots
    // at 1 + k*rec + b*kTraceStamps + i (i = 0..2 phase-specific checkpoints,
    // 3 = done computing, 4 = ns waiting for weight pieces, 5 = pieces not
    // resident when first needed) and CTA 0 finishing the phase at
    // 1 + k*rec + grid*kTraceStamps.
    unsigned long long *trace;
    // Fault injection for tests of the bounded waits (mr_model_inject_fault):
    // the words of phase `withhold_phase` are not published, so its readers'
    // waits run out; -1 = off.
    int withhold_phase;
};

}  // namespace mr
