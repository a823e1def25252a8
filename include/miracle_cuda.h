/*
 * miracle_cuda.h — C ABI of libmiracle_cuda.so, the B200 (sm_100a) engine for
 * the MiracleReasoning token loop.
 *
 * Plain C: opaque handles, plain pointers and sizes, int status codes.  Every
 * call returns MR_OK (0) or an MR_ERR_* code; mr_last_error() then returns a
 * thread-local message.  The Python side (ctypes) raises CUDAError, the
 * counterpart of the reference's OpenCLError (miracle_reasoning/opencl.py:
 * 14-21).  A context (one device, one stream) and everything created from it
 * is used by one host thread at a time, as the reference backend requires
 * (opencl.py:129-133).
 *
 * Two layers:
 *   1. Buffer and kernel entry points with the reference backend's semantics
 *      (opencl.py:178-303, kernels.cl): float32 buffers addressed in ELEMENTS,
 *      bounds-checked copies, and one entry point per reference kernel taking
 *      that kernel's NDRange extents and arguments.  These let the reference's
 *      op-level call sites run unchanged on the GPU.
 *   2. A whole-model engine (mr_model_*) that replaces the reference's Python
 *      per-op dispatch (model.py:257-312) and its LRU weight cache
 *      (weights.py:258-297): weights resident in HBM in their stored dtype,
 *      caches on the device, and one persistent kernel per decode step.
 */
#ifndef MIRACLE_CUDA_H
#define MIRACLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MR_API __attribute__((visibility("default")))
#else
#define MR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MR_ABI_VERSION 1

enum mr_status {
    MR_OK = 0,
    MR_ERR_ARGUMENT = 1,  /* bad shape, offset, name or size: nothing was done */
    MR_ERR_CUDA = 2,      /* a CUDA runtime call failed */
    MR_ERR_STATE = 3,     /* call out of order (e.g. step before finalize) */
    MR_ERR_TIMEOUT = 4,   /* a bounded device-side wait gave up */
    MR_ERR_NOMEM = 5      /* device allocation failed */
};

enum mr_dtype { MR_DTYPE_F32 = 0, MR_DTYPE_F16 = 1, MR_DTYPE_BF16 = 2 };

/* config.py:9-10 FAMILIES, in order */
enum mr_family {
    MR_FAMILY_FLASHNANO_15 = 0,
    MR_FAMILY_FLASHNANO_16 = 1,
    MR_FAMILY_FLASHNANO_17 = 2,
    MR_FAMILY_FLASHLITE_20 = 3,
    MR_FAMILY_FLASHLIGHTING_20 = 4,
    MR_FAMILY_HEAVY_MEDIUM_20 = 5
};

typedef struct mr_context mr_context;
typedef struct mr_buffer mr_buffer;
typedef struct mr_model mr_model;

/* ---- errors, version, devices ------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). */
MR_API const char *mr_last_error(void);
MR_API int mr_abi_version(void);

/* Replaces Device / list_devices (opencl.py:69-115). */
typedef struct {
    int ordinal;
    int sm_count;
    int cc_major, cc_minor;
    uint64_t memory_bytes;
    uint64_t max_allocation_bytes;
    char name[256];
} mr_device_info;

MR_API int mr_device_count(int *count);
MR_API int mr_device_query(int ordinal, mr_device_info *info);

/* ---- context: one device + one stream (OpenCLBackend.__init__, opencl.py:136-166) */
MR_API int mr_context_create(int device_ordinal, mr_context **out);
/* Releases the caller's reference.  Buffers and models made on the context
 * hold their own references, so handles may be released in any order; the
 * stream is destroyed with the last one. */
MR_API int mr_context_destroy(mr_context *ctx);
/* OpenCLBackend.finish (opencl.py:302-303) */
MR_API int mr_context_finish(mr_context *ctx);

/* ---- float32 buffers (opencl.py:178-217) --------------------------------
 * Sizes, offsets and counts are in float32 ELEMENTS.  Upload and download are
 * blocking, like the reference's blocking clEnqueueWrite/ReadBuffer. */
MR_API int mr_buffer_alloc(mr_context *ctx, size_t count, mr_buffer **out);          /* empty()  */
MR_API int mr_buffer_free(mr_buffer *buf);                                           /* Tensor.__del__ */
MR_API int mr_buffer_count(const mr_buffer *buf, size_t *count);
MR_API int mr_buffer_upload(mr_buffer *buf, size_t offset, const float *host, size_t count);   /* upload() */
MR_API int mr_buffer_download(const mr_buffer *buf, size_t offset, float *host, size_t count); /* read() */
/* copy() (opencl.py:209-217): bounds-checked; count 0 is a no-op. */
MR_API int mr_buffer_copy(const mr_buffer *src, mr_buffer *dst, size_t src_offset, size_t dst_offset,
                          size_t count);

/* ---- kernels: one entry per kernels.cl kernel ----------------------------
 * g0/g1 are the NDRange extents the reference passes to run() (opencl.py:
 * 219-239); the remaining arguments are the kernel's, in the kernel's order.
 * Every buffer extent the kernel can touch is checked against its buffer
 * before launch (MR_ERR_ARGUMENT).  All compute in float32 on the device. */
MR_API int mr_op_linear(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *x, const mr_buffer *w,
                        mr_buffer *y, int rows, int out_dim, int in_dim);                /* kernels.cl:5-17 */
MR_API int mr_op_rms(mr_context *ctx, size_t g0, const mr_buffer *x, const mr_buffer *w, mr_buffer *y,
                     int rows, int width, float eps, int affine);                        /* kernels.cl:19-28 */
MR_API int mr_op_rope(mr_context *ctx, size_t g0, const mr_buffer *x, const mr_buffer *freq,
                      const mr_buffer *pos, mr_buffer *y, int rows, int heads, int dim,
                      int split_half);                                                   /* kernels.cl:30-44 */
MR_API int mr_op_swiglu(mr_context *ctx, size_t g0, const mr_buffer *g, const mr_buffer *u, mr_buffer *y,
                        int n);                                                          /* kernels.cl:46-50 */
MR_API int mr_op_axpy(mr_context *ctx, size_t g0, const mr_buffer *x, const mr_buffer *y, mr_buffer *z,
                      int n, float scale);                                               /* kernels.cl:52-56 */
MR_API int mr_op_scores(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *q, const mr_buffer *k,
                        const mr_buffer *extra_k, mr_buffer *s, int heads, int kv_heads, int dim,
                        int capacity, int start, int length, int extra_length);          /* kernels.cl:58-73 */
MR_API int mr_op_softmax(mr_context *ctx, size_t g0, const mr_buffer *x, mr_buffer *y, int rows,
                         int width);                                                     /* kernels.cl:75-84 */
MR_API int mr_op_latent_mask(mr_context *ctx, size_t g0, size_t g1, mr_buffer *scores,
                             const mr_buffer *positions, int heads, int length, int memory,
                             int earliest);                                              /* kernels.cl:86-91 */
MR_API int mr_op_mix(mr_context *ctx, size_t g0, const mr_buffer *p, const mr_buffer *v,
                     const mr_buffer *extra_v, mr_buffer *y, int heads, int kv_heads, int dim,
                     int capacity, int start, int length, int extra_length);             /* kernels.cl:93-107 */
MR_API int mr_op_pool_scores(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *u,
                             const mr_buffer *q, mr_buffer *s, int tokens, int slots,
                             int width);                                                 /* kernels.cl:109-117 */
MR_API int mr_op_pool_mix(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *u, const mr_buffer *p,
                          mr_buffer *z, mr_buffer *anchors, int tokens, int slots, int width,
                          int start_position);                                           /* kernels.cl:119-130 */
MR_API int mr_op_merge_rows(mr_context *ctx, size_t g0, const mr_buffer *x, mr_buffer *y, int width,
                            float a, float b);                                           /* kernels.cl:132-137 */
MR_API int mr_op_block_means(mr_context *ctx, size_t g0, size_t g1, const mr_buffer *x, mr_buffer *y,
                             int length, int width, int block);                          /* kernels.cl:139-148 */

/* ---- whole-model engine --------------------------------------------------
 * Architecture of one model: the fields of ModelConfig (config.py:13-39) that
 * the token loop reads, flattened, plus the per-layer KV head count and window
 * (config.py:83-87) and the float32 inverse-frequency table (config.py:155-197)
 * computed on the host. */
typedef struct {
    int family;            /* enum mr_family */
    int vocab_size, hidden_size, layers, query_heads, kv_heads, head_dim, ffn_dim;
    int context_length;    /* MiracleModel(context_length=...) (model.py:43-53) */
    int window;            /* 0 = none */
    int tie_embeddings, qk_norm, split_half_rope;
    float norm_eps, residual_scale, cbr_norm_eps;
    int latent_dim, memory_slots, cbr_chunk_size, cbr_slots, inner_loop_steps;
    /* heavy-medium-2.0 (config.source, model.py:192-255) */
    int routed_experts, router_groups, router_top_k_min, router_top_k_max, shared_experts;
    int block_size, global_slots;
    float router_temperature;   /* already max(T, 1e-4) */
    float alibi_slope;          /* float32(alibi_slope_scale / sqrt(head_dim)) */
} mr_model_config;

/* Allocates the model description; no weights yet.  (MiracleModel.__init__,
 * model.py:43-56.)  layer_kv_heads[layers], layer_window[layers] (0 = full
 * history), inv_freq[head_dim/2]. */
MR_API int mr_model_create(mr_context *ctx, const mr_model_config *config, const int *layer_kv_heads,
                           const int *layer_window, const float *inv_freq, mr_model **out);
MR_API int mr_model_destroy(mr_model *model);

/* Copies one tensor's STORED bytes (dtype F32/F16/BF16, row-major) to HBM.
 * name is the canonical name of weights.py expected_shapes (e.g.
 * "layers.3.ffn.gate"); its shape must match.  Replaces WeightCache.tensor
 * (weights.py:266-280): no widening, no eviction.  The caller keeps ownership
 * of the host memory. */
MR_API int mr_model_load_tensor(mr_model *model, const char *name, int dtype, int ndim,
                                const int64_t *shape, const void *host);

/* The same, read by the library straight from a checkpoint file: `bytes of
 * the tensor` starting at byte `offset` of the file at `path` (a safetensors
 * data span), through two page-locked 64 MB buffers, each read (pread) while
 * the other is copied to HBM.  Nothing is widened or held on the host.
 * Replaces the reference's mmap + widening read of a safetensors tensor
 * (weights.py:58-61, 64-74) on the way to HBM residency. */
MR_API int mr_model_load_file(mr_model *model, const char *name, int dtype, int ndim, const int64_t *shape,
                              const char *path, uint64_t offset);
/* Synthetic benchmark weights generated on the device (no host copy): BF16
 * values of the counter-hash generator of synthetic.py (seed, tensor_index,
 * scale = float32(std / 65536)); scale 0 fills every element with fill.  No
 * reference counterpart (the reference loads checkpoints only). */
MR_API int mr_model_fill_synthetic(mr_model *model, const char *name, int dtype, int ndim,
                                   const int64_t *shape, uint64_t seed, int tensor_index, float scale,
                                   float fill);
/* Checks that every tensor is present, allocates caches and builds the decode plan. */
MR_API int mr_model_finalize(mr_model *model);
/* model.reset() (model.py:74-77): position 0, caches emptied, failure cleared. */
MR_API int mr_model_reset(mr_model *model);

/* Prompts of two or more tokens run batched (tensor-core GEMMs, causal
 * attention over the chunk) when every projection and the lm_head are BF16;
 * otherwise, or with enable = 0, token by token through the decode kernel
 * (the reference's serial order, model.py:295-312).  enable = 1: GEMMs on
 * tcgen05 (default); enable = 2: on mma.sync (the legacy tensor-core path,
 * kept as a comparison baseline).  *available (optional) reports whether the
 * batched path applies to this model. */
MR_API int mr_model_set_batched_prefill(mr_model *model, int enable, int *available);

/* Tensor-parallel decode over `ranks` GPUs, one process per GPU (reference:
 * the token loop of model.py:257-285, each projection and the lm_head split
 * by output row, attention by KV head).  Call mr_model_set_tensor_parallel
 * before mr_model_finalize; then every rank exports its exchange arena
 * (mr_model_tp_handle: a CUDA IPC handle, bytes >= 64), the handles are
 * exchanged (any host channel), and mr_model_tp_connect maps the others'
 * arenas (handles: ranks x bytes_each, in rank order).  Every rank then makes
 * the same calls in the same order; each step's words are stored into every
 * rank's arena over NVLink and the argmax is agreed at the step end.  KV head
 * counts must divide by `ranks`. */
MR_API int mr_model_set_tensor_parallel(mr_model *model, int rank, int ranks);
MR_API int mr_model_tp_handle(mr_model *model, void *handle, size_t bytes);
MR_API int mr_model_tp_connect(mr_model *model, const void *handles, size_t bytes_each);
MR_API int mr_model_position(const mr_model *model, int *position);
MR_API int mr_model_weight_bytes(const mr_model *model, uint64_t *bytes);

/* One token (model.py:257-285 plus the head at 307-308).  logits_out
 * (vocab floats, host) and/or argmax_out may be NULL.  Fails with
 * MR_ERR_ARGUMENT if the token is out of vocabulary or the context is full. */
MR_API int mr_model_step(mr_model *model, int token, float *logits_out, int *argmax_out);
/* model.prefill (model.py:295-312): n tokens; out receives the last token's
 * logits (return_all = 0, vocab floats) or every token's (n * vocab floats). */
MR_API int mr_model_prefill(mr_model *model, const int *ids, int n, int return_all, float *out);
/* Greedy generation on the device (model.py:318-357 with temperature 0):
 * prefill, then up to max_new tokens chosen by device argmax (lowest index
 * among equal maxima, as numpy.argmax), stopping after eos.  Writes the
 * generated ids to out_tokens and their number to out_count.  A non-finite
 * logit sets *out_nonfinite and stops. */
MR_API int mr_model_generate_greedy(mr_model *model, const int *ids, int n, int max_new, int eos,
                                    int *out_tokens, int *out_count, int *out_nonfinite);
/* Seeded sampling on the device (reference: generate with temperature > 0,
 * model.py:318-357 and the sampling procedure of model.py:343-352): the prompt,
 * then per token the stable descending order of the logits, float64
 * softmax at `temperature` over the top_k (0: all), the top_p cutoff and
 * NumPy Generator.choice, every sum in NumPy's order, the draws from the PCG64
 * state of numpy.random.default_rng(seed) given as pcg_state[4] = {state >> 64,
 * state & (2^64-1), inc >> 64, inc & (2^64-1)}.  temperature 0 takes the argmax.
 * Stops after eos or max_new tokens; *out_nonfinite = 1 when a non-finite
 * logit stopped it (the reference raises there).  One GPU. */
MR_API int mr_model_generate_sampled(mr_model *model, const int *ids, int n, int max_new, int eos, double temperature,
                                     int top_k, double top_p, const uint64_t *pcg_state, int *out_tokens,
                                     int *out_count, int *out_nonfinite);

/* Cache state of one layer (and inner loop for heavy-medium-2.0), mirroring
 * what the reference keeps in MiracleModel.states (model.py:15-33, 104-190). */
typedef struct {
    int present;           /* 0 until the layer has seen a token (lazy state in the reference) */
    int ring_count, ring_capacity, ring_length, ring_start;
    int relay_count;       /* flashnano-1.6 CBR rows */
    int latent_rows, memory_size;   /* flashlighting-2.0 */
} mr_layer_state;
MR_API int mr_model_layer_state(const mr_model *model, int layer, int loop, mr_layer_state *out);
/* flashlighting-2.0: positions of the latent rows (rows ints) of one layer. */
MR_API int mr_model_latent_positions(const mr_model *model, int layer, int *out, int capacity, int *rows);
/* flashlighting-2.0: how many tokens each latent row stands for (rows floats;
 * memory rows first, as the reference's state["counts"], model.py:183-185). */
MR_API int mr_model_latent_counts(const mr_model *model, int layer, float *out, int capacity, int *rows);
/* Discrete decisions of the LAST step, for parity tests:
 * heavy top-k:  blocks[heads * global_slots], -1 padded, ascending per head;
 * MoE:          experts[router_top_k_max] (-1 padded, rank order), weights[...] */
MR_API int mr_model_last_topk(const mr_model *model, int layer, int loop, int *blocks, int capacity);
MR_API int mr_model_last_experts(const mr_model *model, int layer, int loop, int *experts,
                                 float *weights, int capacity);
/* heavy-medium-2.0: float32 log1p(d) for d = 0 .. context_length-1, computed by
 * the host (the reference's distance penalty applies NumPy's float32 log1p,
 * model.py:221-222).  Required before the first token. */
MR_API int mr_model_set_log1p_table(mr_model *model, const float *values, int n);

/* Benchmark helper: run `steps` greedy decode steps back to back on the
 * device (each step's token = previous argmax), starting from the current
 * state; returns device milliseconds measured with CUDA events on the engine's
 * stream.  No reference counterpart. */
MR_API int mr_model_bench_decode(mr_model *model, int first_token, int steps, float *device_ms);

/* Resident tensors of a finalized model, for the families whose token step
 * runs on the host over the op kernels (flashnano-1.6, FlashLighting, Heavy
 * Medium; the decode engine covers the grouped-query families).  They replace
 * the reference's WeightCache (weights.py:258-297): the weights stay in HBM in
 * their stored dtype.
 *   mr_model_linear: y[rows, out] = x[rows, in] . W^T, W = the named tensor;
 *     the reference's linear arithmetic (kernels.cl:5-17) over the exactly
 *     widened weights, so bit-identical to it.
 *   mr_model_tensor_rows: rows [row0, row0 + nrows) widened to float32 into
 *     `out` (a 1-D tensor is one row).
 *   mr_model_tensor_download: the whole tensor widened to float32 on the host. */
MR_API int mr_model_linear(mr_model *model, const char *name, const mr_buffer *x, int rows, mr_buffer *y);
MR_API int mr_model_tensor_rows(mr_model *model, const char *name, int64_t row0, int64_t nrows, mr_buffer *out);
MR_API int mr_model_tensor_download(mr_model *model, const char *name, float *host, size_t count);

/* Tracing: run one decode step (feeding `token`) with per-phase device
 * timestamps (globaltimer, ns).  Layout: stamps[0] = launch start; the k-th
 * executed phase has a record of grid*6 + 1 stamps at 1 + k*(grid*6 + 1):
 * CTA b's slots at offset b*6 + i (i = 0..2 phase-specific checkpoints, 3 =
 * done computing, 4 = ns spent waiting for weight pieces, 5 = pieces not yet
 * in shared memory when first needed) and CTA 0 finishing the phase at
 * offset grid*6 (phases are not separated by grid barriers; each CTA moves
 * on when its own inputs have arrived).  GEMV checkpoints: input loaded,
 * input normalised, weights consumed; attention: first tile and q/k/v
 * loaded, q/k prepared, scores/mix done; slot 3: phase done.  A CTA with no
 * work in a phase leaves slots 0-2 zero.
 * *phases receives the number of executed phases, *grid the CTA count.
 * heavy-medium-2.0 (a sequence of kernel launches, not one persistent
 * kernel): stamps[0] = the step's start, stamps[k] = the time the step's k-th
 * kernel had completed, *phases = the number of kernels, *grid = 0; when
 * capacity leaves room, the last 8 * P stamps hold 8 probes for each of the P
 * = 6 * layers * inner loops + 1 projection / attention / router launches
 * (first CTA start, first CTA past its dependency wait, last CTA done staging,
 * last CTA done with its main loop, last CTA exit; 3 unused).  No
 * reference counterpart (the reference has no tracing). */
MR_API int mr_model_trace_decode(mr_model *model, int token, uint64_t *stamps, int capacity, int *phases,
                                 int *grid);

/* Bounded device waits: every wait of the model's kernels on another CTA's or
 * another rank's data (exchange words, counters, copies in flight) gives up
 * after `nanoseconds` (default 2 s, at least 1 ms), records an error, and the
 * call returns MR_ERR_TIMEOUT; the model then refuses further steps until
 * mr_model_reset (the reference latches _failed, model.py:298-311).  The
 * setting survives mr_model_reset.  No reference counterpart (the reference
 * has no device-side waits). */
MR_API int mr_model_set_wait_limit(mr_model *model, uint64_t nanoseconds);

/* Fault injection for tests of that path, on the host's side: with phase >= 0
 * the decode kernel does not publish the words of step phase `phase` (Heavy
 * Medium: the attention units do not count their key / value rows), so the
 * readers' bounded waits run out; -1 turns it off.  No GPU fault is involved.
 * No reference counterpart. */
MR_API int mr_model_inject_fault(mr_model *model, int phase);

/* Attention that allocates nothing on the device.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc while they run
 * (a framework that owns all device memory through its own pool, or code in a
 * section where an allocation could synchronise the device or fail).  Same
 * result, bit for bit, as CUDABackend.attention / mr_op_scores + mr_op_softmax
 * + mr_op_mix (the same per-score dot products, the softmax denominator summed
 * in row order, the value mix in row order), but the [heads x (length +
 * extra_length)] score matrix
 * lives in a 4 MiB file-scope device array that every GPU loading this library
 * keeps until the process exits.  All pointers are device pointers the caller
 * owns; keys/values are ring buffers [capacity, kv_heads*dim] read in logical
 * order [start, start+length) (64-bit row arithmetic: any start >= 0 is
 * valid), then extra rows [extra_length, kv_heads*dim]; with length 0 the
 * ring pointers may be NULL and capacity 0.
 * heads * (length + extra_length) above 1048576 fails with MR_ERR_ARGUMENT.
 * The first call on a device looks up the array's address (do it before any
 * stream capture); every call shares the array, so calls that overlap on the
 * GPU race and must be serialised by the caller.  Runs on ctx's stream. */
MR_API int mr_attention_static_scratch(mr_context *ctx, const float *q, const float *keys, const float *values,
                                       const float *extra_keys, const float *extra_values, float *out, int heads,
                                       int kv_heads, int dim, int capacity, int start, int length,
                                       int extra_length);

#ifdef __cplusplus
}
#endif
#endif /* MIRACLE_CUDA_H */
