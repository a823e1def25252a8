// Persistent decode kernel: one cooperative launch per token, one CTA per SM,
// every phase of the step separated by a bounded grid barrier.
//
// Reference semantics per phase:
//   GEMV      model._linear / kernels.cl linear (5-17), RMSNorm of the input
//             (kernels.cl rms, 19-28), residual axpy (52-56), SwiGLU (46-50)
//   ATTN_GQA  model._gqa (model.py:95-116): per-head Q/K RMSNorm, RoPE
//             (kernels.cl:30-44), ring append (model.py:21-25), scores /
//             softmax / mix over the ring in logical order plus relay rows
//             (kernels.cl:58-107), split over key chunks; the chunks are
//             merged (softmax-rescaled) by the next GEMV phase as it loads
//             its input.
//
// CTA layout: warps 0-14 compute (they synchronise among themselves with
// named barrier 1, never with __syncthreads), warp 15 is the weight-stream
// producer.  The producer walks the CTA's piece table (engine.cuh) and issues
// TMA bulk copies (cp.async.bulk) into a shared-memory byte ring, each piece
// completing a "full" mbarrier; the compute warps consume the pieces in the
// same order -- they derive the order from the phase list, so only the ring
// offset passes between the two sides -- and return each slot through an
// "empty" mbarrier.  The producer runs ahead across phases and grid barriers
// as far as the ring has room, so a phase normally finds its weights already
// in shared memory.
//
// All waits are bounded (2 s): a wait that gives up records an error code in
// StepState, the compute warps stop, the producer waits (bounded) for its
// copies in flight, and the host raises.
//
// Numerics: weights are widened from their stored dtype exactly as the
// reference widens them; all arithmetic is float32.  Dot products and the
// softmax use tree/online reductions, so logits match the reference within
// float32 rounding (the parity tests pin atol 2e-5 / rtol 2e-4), not bit for
// bit.  Element-wise steps (residual, SwiGLU, RoPE) round each product and sum
// separately, as FP_CONTRACT OFF does in the reference.
#include "engine.cuh"

namespace mr {
namespace {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr int kMaxHeadDim = 128;

// Fixed part of the dynamic shared memory; the scratch floats and the weight
// ring follow it.
struct Control {
    unsigned long long full[kQueue];   // piece landed (producer expect_tx + bulk-copy bytes)
    unsigned long long empty[kQueue];  // piece consumed (compute thread 0 arrives)
    Phase phase[2];                    // current and next phase descriptor
    int offset[kQueue];                // ring offset of each piece in flight (producer writes)
    float partial[kEngineWarps * kEngineWarps];
    float y[2][kRowBatch];             // dot products of alternate pieces
    float gate[kRowBatch];             // SwiGLU gate rows of the current row batch
    float xres[kRowBatch];             // this CTA's rows of the residual stream, for the whole launch
    float gains[2 * kMaxHeadDim];      // attention q / k norm gains
    float rope_cos[kMaxHeadDim / 2];   // RoPE cos / sin of this launch's position, per frequency
    float rope_sin[kMaxHeadDim / 2];
    GroupTable group[2][2];            // piece-group tables: [phase parity][group parity]
    int2 rowinfo[2][kRowBatch];        // row tables of alternate groups (build_rows)
    float red[kEngineWarps];
    unsigned long long best[kEngineWarps];
    int ok;
    int ranks;                         // tensor-parallel ranks (1: single GPU)
    char *arena;                       // this rank's exchange arena
    char *peers[kMaxRanks];            // every rank's arena (exchange stores go to all)
    int abort;                         // the compute warps stopped: the producer stops too
    unsigned long long wait_ns;        // tracing: time thread 0 spent in take_piece this phase
    int late;                          // tracing: pieces not resident at their first probe
    int withhold;                      // fault injection: words tagged withhold_tag are not stored
    unsigned withhold_tag;
};

// How long a bounded wait may last (mr_model_set_wait_limit; default 2 s).
__device__ __forceinline__ unsigned long long wait_limit(const StepState *st) {
    const unsigned long long v = *reinterpret_cast<volatile const unsigned long long *>(&st->wait_limit_ns);
    return v ? v : kWaitLimitNs;
}

struct StepInfo {
    int position, token, logits_row;
    unsigned tag_base;  // exchange tag of phase p: tag_base + p
    int xr0, xr1;       // this CTA's rows of the residual stream (kept in Control::xres)
};

// ---- compute-warp synchronisation (named barrier 1, the compute threads) --------------
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kEngineThreads) : "memory"); }
// Barrier that also ANDs a predicate over the compute threads.
__device__ __forceinline__ bool csync_and(bool v) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.s32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(static_cast<int>(v)), "n"(kEngineThreads)
        : "memory");
    return r != 0;
}

// Phase trace checkpoints (no-ops unless the launch carries a trace buffer).
struct Tracer {
    unsigned long long *rec;  // this phase's record, or NULL
    __device__ void mark(int i) const {
        if (!rec) return;
        csync();
        if (threadIdx.x == 0) rec[blockIdx.x * kTraceStamps + i] = global_ns();
    }
    // Slots 4 and 5: weight-piece waiting of the phase (thread 0's accounting).
    __device__ void waits(unsigned long long &wait_ns, int &late) const {
        if (!rec || threadIdx.x != 0) return;
        rec[blockIdx.x * kTraceStamps + 4] = wait_ns;
        rec[blockIdx.x * kTraceStamps + 5] = static_cast<unsigned long long>(late);
        wait_ns = 0;
        late = 0;
    }
};

struct Smem {
    Control *c;
    float *scratch;
    float *attn;        // attention region of the scratch
    unsigned char *ring;
    int ring_bytes;
};


__device__ __forceinline__ int esize(int dtype) { return dtype == MR_DTYPE_F32 ? 4 : 2; }

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- asynchronous copies into shared memory ----------------------------------------------
// Data written earlier in the same launch by other CTAs is read through L2
// only (.cg, 16-byte granules); .ca (4-byte) is used only for data written by
// earlier launches.
__device__ __forceinline__ void cp_async16_cg(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

// ---- exchange words (see engine.cuh) --------------------------------------------------
// Readers poll at system scope: with tensor parallelism the words of a phase
// are stored into this GPU's memory by every rank's GPU.
__device__ __forceinline__ Word ld_word(const Word *p) {
    Word v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// A word only this GPU reads (attention chunk partials).
__device__ __forceinline__ void st_word(Word *p, float v, unsigned tag) {
    const Word w = (static_cast<Word>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_word_sys(Word *p, Word w) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ bool word_ok(Word w, unsigned tag) { return static_cast<unsigned>(w >> 32) == tag; }
__device__ __forceinline__ float word_value(Word w) { return __uint_as_float(static_cast<unsigned>(w)); }

// The same offset of another rank's arena.
template <typename T>
__device__ __forceinline__ T *peer_ptr(const Control &c, int j, T *p) {
    return reinterpret_cast<T *>(c.peers[j] + (reinterpret_cast<char *>(p) - c.arena));
}
// A word every rank reads: stored into every rank's arena (NVLink peer
// stores for the others) when tensor parallel.
__device__ __forceinline__ void st_word_all(const Control &c, Word *p, float v, unsigned tag) {
    if (c.withhold && tag == c.withhold_tag) return;  // an injected fault: this phase publishes nothing
    if (c.ranks == 1) {
        st_word(p, v, tag);
        return;
    }
    const Word w = (static_cast<Word>(tag) << 32) | __float_as_uint(v);
    for (int j = 0; j < c.ranks; ++j) st_word_sys(peer_ptr(c, j, p), w);
}

// ---- mbarrier / bulk copy primitives --------------------------------------------------
__device__ __forceinline__ void mbar_init(unsigned long long *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long *bar, int parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or the hint elapses) instead of re-polling and taking issue
// slots from the compute warps of its sub-partition.
__device__ __forceinline__ bool mbar_wait_sleep(unsigned long long *bar, int parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(unsigned long long *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// L2 policy of the weight stream: read once per step and far larger than L2,
// it is evicted first, so that what is re-read every step (key/value rings, the
// plan's records, exchange words) stays in L2 across steps.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, unsigned long long *bar,
                                          uint64_t policy) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Bounded wait on one phase of an mbarrier.  Gives up when another wait has
// already recorded an error, when the compute warps stopped (`watch_abort`),
// or after wait_limit(st) (recording 1000 + phase).
__device__ bool wait_bar(unsigned long long *bar, int parity, StepState *st, const Control &c, int phase,
                         bool watch_abort) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t start = 0;
    for (unsigned spin = 0;; ++spin) {
        if (mbar_wait_sleep(bar, parity)) return true;
        if ((spin & 7u) == 7u) {
            if (*reinterpret_cast<volatile const int *>(&st->error)) return false;
            if (watch_abort && *reinterpret_cast<volatile const int *>(&c.abort)) return false;
            const uint64_t now = global_ns();
            if (!start) {
                start = now;
            } else if (now - start > wait_limit(st)) {
                atomicCAS(&st->error, 0, 1000 + phase);
                return false;
            }
        }
    }
}

// Reads N exchange words at addr(0) .. addr(N - 1) (NULL: none), polling each
// until it carries its tag (tag_of(u); read_words: one tag for all);
// bounded like every wait (gives up early when another wait recorded an error).  Every load is issued before the first
// check; addresses are recomputed rather than held, to spare registers.
template <int N, typename Addr, typename TagOf>
__device__ __forceinline__ bool read_words_tagged(Addr addr, TagOf tag_of, float (&out)[N], StepState *st,
                                                  int phase) {
    Word w[N];
#pragma unroll
    for (int u = 0; u < N; ++u) {
        const Word *src = addr(u);
        w[u] = src ? ld_word(src) : (static_cast<Word>(tag_of(u)) << 32);
    }
    uint64_t start = 0;
    for (unsigned spin = 0;; ++spin) {
        bool all = true;
#pragma unroll
        for (int u = 0; u < N; ++u)
            if (!word_ok(w[u], tag_of(u))) {
                all = false;
                w[u] = ld_word(addr(u));
            }
        if (all) break;
        if ((spin & 15u) == 15u) {
            if (*reinterpret_cast<volatile const int *>(&st->error)) return false;
            const uint64_t now = global_ns();
            if (!start) {
                start = now;
            } else if (now - start > wait_limit(st)) {
                atomicCAS(&st->error, 0, 1000 + phase);
                return false;
            }
        }
    }
#pragma unroll
    for (int u = 0; u < N; ++u) out[u] = word_value(w[u]);
    return true;
}
template <int N, typename Addr>
__device__ __forceinline__ bool read_words(Addr addr, unsigned tag, float (&out)[N], StepState *st, int phase) {
    return read_words_tagged(addr, [tag](int) { return tag; }, out, st, phase);
}

// ---- the weight-stream producer (lane 0 of warp 16) -----------------------------------
__device__ __forceinline__ uint4 ld_desc(const PieceDesc *table, int i, int count) {
    if (i >= count) return make_uint4(0u, 0u, 0u, 0u);
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(table + i));
    return v;
}

// Issues every piece of this CTA's stream (up to the head phase when no
// logits are needed) into the ring, allocating ring bytes first-fit in
// stream order: a piece goes after the newest one, or wraps to offset 0, once
// the pieces it would overwrite have been consumed.  Descriptors are loaded
// four pieces ahead.  Before returning, waits (bounded) until every issued
// copy has landed, so that no copy writes shared memory after the CTA exits.
__device__ void produce(const StepControl &ctl, bool need_head, int head_phase, StepState *st, const Smem &sm) {
    Control &c = *sm.c;
    const PieceDesc *table = ctl.pieces + static_cast<size_t>(blockIdx.x) * ctl.piece_stride;
    const int count = ctl.piece_count[blockIdx.x];
    uint4 q0 = ld_desc(table, 0, count), q1 = ld_desc(table, 1, count), q2 = ld_desc(table, 2, count),
          q3 = ld_desc(table, 3, count);
    int tail = 0, head_off = 0, issued = 0;
    bool ok = true;
    const uint64_t policy = l2_evict_first();
    while (ok && issued < count) {
        const uint4 d = q0;
        q0 = q1;
        q1 = q2;
        q2 = q3;
        q3 = ld_desc(table, issued + 4, count);
        const void *src = reinterpret_cast<const void *>((static_cast<unsigned long long>(d.y) << 32) | d.x);
        const int bytes = static_cast<int>(d.z), phase = static_cast<int>(d.w);
        if (!need_head && phase == head_phase) break;
        // a free mbarrier slot: piece issued - kQueue must have been consumed
        while (ok && tail <= issued - kQueue) {
            ok = wait_bar(&c.empty[tail % kQueue], (tail / kQueue) & 1, st, c, phase, true);
            ++tail;
        }
        int off = 0;
        while (ok) {
            if (tail == issued) {  // nothing in flight: the ring is empty
                off = 0;
                break;
            }
            const int tail_off = c.offset[tail % kQueue];
            if (head_off > tail_off) {
                if (head_off + bytes <= sm.ring_bytes) {
                    off = head_off;
                    break;
                }
                if (bytes <= tail_off) {
                    off = 0;
                    break;
                }
            } else if (head_off < tail_off && head_off + bytes <= tail_off) {
                off = head_off;
                break;
            }
            ok = wait_bar(&c.empty[tail % kQueue], (tail / kQueue) & 1, st, c, phase, true);
            ++tail;
        }
        if (!ok) break;
        const int slot = issued % kQueue;
        c.offset[slot] = off;
        // the region was last read through the generic proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bulk_load(sm.ring + off, src, static_cast<uint32_t>(bytes), &c.full[slot], policy);
        head_off = off + bytes;
        ++issued;
    }
    const uint64_t start = global_ns();
    for (int j = max(tail, issued - kQueue); j < issued; ++j) {
        while (!mbar_wait_sleep(&c.full[j % kQueue], (j / kQueue) & 1))
            if (global_ns() - start > wait_limit(st)) return;
    }
}

// Warp 0: bounded wait until pieces [first, first + count) are in the ring,
// lane k watching piece k (count <= kGroupPieces), so the checks overlap.
// The compute barrier that follows orders the bulk-copy writes, observed
// here, before every thread's reads of the ring.  With `tracing`, thread 0
// accounts the waiting time and the pieces not yet landed.
__device__ bool wait_group(Control &c, int first, int count, StepState *st, int phase, bool tracing) {
    const int lane = threadIdx.x & 31;
    const uint64_t t0 = tracing && lane == 0 ? global_ns() : 0;
    bool ok = true, late = false;
    if (lane < count) {
        unsigned long long *bar = &c.full[(first + lane) % kQueue];
        const int parity = ((first + lane) / kQueue) & 1;
        if (tracing) late = !mbar_try_wait(bar, parity);
        ok = wait_bar(bar, parity, st, c, phase, false);
    }
    ok = __all_sync(0xffffffffu, ok);
    if (tracing) {
        const int n_late = __popc(__ballot_sync(0xffffffffu, late));
        if (lane == 0) {
            c.late += n_late;
            c.wait_ns += global_ns() - t0;
        }
    }
    return ok;
}

// ---- grid barrier ------------------------------------------------------------------
// Release-add arrival (cumulative over the CTA's writes ordered by the compute
// barrier), acquire polling by thread 0, bounded by wait_limit(st).  `during`
// runs in every compute thread after the arrival, overlapping the wait.
template <typename During>
__device__ bool grid_barrier(StepState *st, unsigned long long target, int phase, Control &c, During during) {
    csync();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(&st->barrier) : "memory");
    during();
    if (threadIdx.x == 0) {
        int ok = 1;
        uint64_t start = 0;
        for (unsigned spin = 0;; ++spin) {
            if (ld_acquire_u64(&st->barrier) >= target) break;
            if ((spin & 63u) == 63u) {
                if (*reinterpret_cast<volatile int *>(&st->error)) {
                    ok = 0;
                    break;
                }
                const uint64_t now = global_ns();
                if (!start) {
                    start = now;
                } else if (now - start > wait_limit(st)) {
                    atomicCAS(&st->error, 0, 1000 + phase);
                    ok = 0;
                    break;
                }
            }
        }
        c.ok = ok;
        if (!ok) c.abort = 1;
    }
    csync();
    return c.ok != 0;
}

// Block sum in a fixed order (identical bits in every thread and CTA).  The
// caller separates two calls by at least one compute barrier.
__device__ float block_sum(float v, Control &c) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) c.red[warp] = v;
    csync();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kEngineWarps; ++w) total += c.red[w];
    return total;
}

// ---- dot products -------------------------------------------------------------------
// The input vector x of a GEMV phase, as staged in shared memory.  Weights are
// read in 16-byte chunks (8 BF16/F16 or 4 F32 columns).  For 16-bit weights in
// the ring, x is stored split ("lo" plane: columns 8c..8c+3 of chunk c at
// lo + 4c; "hi" plane: 8c+4..8c+7 at hi + 4c), so that a warp reading the
// chunks lane, lane + 32, ... loads consecutive 16-byte blocks (no bank
// conflict); otherwise x is plain (lo = x, hi = x + 4, stride 8 or 4).
struct XView {
    const float *lo, *hi, *plain;
    int stride;
    __device__ __forceinline__ float4 L(int c) const { return *reinterpret_cast<const float4 *>(lo + c * stride); }
    __device__ __forceinline__ float4 H(int c) const { return *reinterpret_cast<const float4 *>(hi + c * stride); }
};
__device__ __forceinline__ XView x_split(const float *in, int cols) { return XView{in, in + cols / 2, nullptr, 4}; }
__device__ __forceinline__ XView x_plain(const float *in, int dtype) {
    return dtype == MR_DTYPE_F32 ? XView{in, in, in, 4} : XView{in, in + 4, in, 8};
}
// Position of column j of x in the split layout.
__device__ __forceinline__ int split_index(int j, int cols) { return (j >> 3) * 4 + (j & 3) + ((j & 4) ? cols / 2 : 0); }

template <int DT>
struct RowDot;

// One 16-byte chunk of weights times its x values, added column by column to
// running sums s[0 .. VEC-1] (independent FMAs: a chain per chunk left the
// warps waiting on FMA latency); fold() sums them pairwise.
template <>
struct RowDot<MR_DTYPE_BF16> {
    static constexpr int VEC = 8;
    __device__ static void add(float (&s)[VEC], const uint4 &w, const float4 a, const float4 b) {
        s[0] = fmaf(__uint_as_float(w.x << 16), a.x, s[0]);
        s[1] = fmaf(__uint_as_float(w.x & 0xffff0000u), a.y, s[1]);
        s[2] = fmaf(__uint_as_float(w.y << 16), a.z, s[2]);
        s[3] = fmaf(__uint_as_float(w.y & 0xffff0000u), a.w, s[3]);
        s[4] = fmaf(__uint_as_float(w.z << 16), b.x, s[4]);
        s[5] = fmaf(__uint_as_float(w.z & 0xffff0000u), b.y, s[5]);
        s[6] = fmaf(__uint_as_float(w.w << 16), b.z, s[6]);
        s[7] = fmaf(__uint_as_float(w.w & 0xffff0000u), b.w, s[7]);
    }
};

template <>
struct RowDot<MR_DTYPE_F16> {
    static constexpr int VEC = 8;
    __device__ static void add(float (&s)[VEC], const uint4 &w, const float4 a, const float4 b) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&w);
        const float2 p0 = __half22float2(h[0]), p1 = __half22float2(h[1]), p2 = __half22float2(h[2]),
                     p3 = __half22float2(h[3]);
        s[0] = fmaf(p0.x, a.x, s[0]);
        s[1] = fmaf(p0.y, a.y, s[1]);
        s[2] = fmaf(p1.x, a.z, s[2]);
        s[3] = fmaf(p1.y, a.w, s[3]);
        s[4] = fmaf(p2.x, b.x, s[4]);
        s[5] = fmaf(p2.y, b.y, s[5]);
        s[6] = fmaf(p3.x, b.z, s[6]);
        s[7] = fmaf(p3.y, b.w, s[7]);
    }
};

template <>
struct RowDot<MR_DTYPE_F32> {
    static constexpr int VEC = 4;
    __device__ static void add(float (&s)[VEC], const uint4 &w, const float4 a, const float4) {
        s[0] = fmaf(__uint_as_float(w.x), a.x, s[0]);
        s[1] = fmaf(__uint_as_float(w.y), a.y, s[1]);
        s[2] = fmaf(__uint_as_float(w.z), a.z, s[2]);
        s[3] = fmaf(__uint_as_float(w.w), a.w, s[3]);
    }
};

template <int DT>
__device__ __forceinline__ float fold(const float (&s)[RowDot<DT>::VEC]) {
    float t = (s[0] + s[1]) + (s[2] + s[3]);
    if constexpr (RowDot<DT>::VEC == 8) t = t + ((s[4] + s[5]) + (s[6] + s[7]));
    return t;
}

template <int DT>
__device__ __forceinline__ void xadd(float (&s)[RowDot<DT>::VEC], const uint4 &w, const XView &x, int c) {
    RowDot<DT>::add(s, w, x.L(c), DT == MR_DTYPE_F32 ? float4{} : x.H(c));
}

// Weights read straight from global memory (non-bulk phases): bypass L1.
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_smem(const uint4 *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_addr(p)));
    return v;
}

// Partial dot product of one row (16-byte chunks first, first+stride, ...).
// FROM_SMEM rows are in the weight ring (always whole 16-byte chunks); global
// rows may have a scalar tail, taken by `tail_lane` (-1: none), and rows whose
// byte length is not a multiple of 16 use scalar loads only (plain x).
template <int DT, bool FROM_SMEM>
__device__ float row_partial(const char *rp, int cols, int first, int stride, int tail_lane, const XView &x) {
    using D = RowDot<DT>;
    const int nv = cols / D::VEC;
    const size_t row_bytes = static_cast<size_t>(cols) * esize(DT);
    // a running sum per column of a chunk; four chunks' loads in flight at a time
    float acc = 0.f;
    float sums[D::VEC];
#pragma unroll
    for (int k = 0; k < D::VEC; ++k) sums[k] = 0.f;
    if (FROM_SMEM || (row_bytes & 15) == 0) {
        const uint4 *v = reinterpret_cast<const uint4 *>(rp);
        int c = first;
        for (; c + 3 * stride < nv; c += 4 * stride) {
            uint4 w0, w1, w2, w3;
            if (FROM_SMEM) {
                w0 = ld_smem(v + c), w1 = ld_smem(v + c + stride), w2 = ld_smem(v + c + 2 * stride),
                w3 = ld_smem(v + c + 3 * stride);
            } else {
                w0 = ld_stream(v + c), w1 = ld_stream(v + c + stride), w2 = ld_stream(v + c + 2 * stride),
                w3 = ld_stream(v + c + 3 * stride);
            }
            xadd<DT>(sums, w0, x, c);
            xadd<DT>(sums, w1, x, c + stride);
            xadd<DT>(sums, w2, x, c + 2 * stride);
            xadd<DT>(sums, w3, x, c + 3 * stride);
        }
        if (c + stride < nv) {
            const uint4 w0 = FROM_SMEM ? ld_smem(v + c) : ld_stream(v + c);
            const uint4 w1 = FROM_SMEM ? ld_smem(v + c + stride) : ld_stream(v + c + stride);
            xadd<DT>(sums, w0, x, c);
            xadd<DT>(sums, w1, x, c + stride);
            c += 2 * stride;
        }
        for (; c < nv; c += stride) xadd<DT>(sums, FROM_SMEM ? ld_smem(v + c) : ld_stream(v + c), x, c);
        acc = fold<DT>(sums);
        if (!FROM_SMEM && tail_lane >= 0)
            for (int j = nv * D::VEC + tail_lane; j < cols; j += 32) acc = fmaf(load_weight(rp, DT, j), x.plain[j], acc);
    } else if (tail_lane >= 0) {
        for (int j = tail_lane; j < cols; j += 32) acc = fmaf(load_weight(rp, DT, j), x.plain[j], acc);
    }
    return acc;
}

template <bool FROM_SMEM>
__device__ float row_partial_any(int dtype, const char *rp, int cols, int first, int stride, int tail_lane,
                                 const XView &x) {
    switch (dtype) {
        case MR_DTYPE_BF16: return row_partial<MR_DTYPE_BF16, FROM_SMEM>(rp, cols, first, stride, tail_lane, x);
        case MR_DTYPE_F16: return row_partial<MR_DTYPE_F16, FROM_SMEM>(rp, cols, first, stride, tail_lane, x);
        default: return row_partial<MR_DTYPE_F32, FROM_SMEM>(rp, cols, first, stride, tail_lane, x);
    }
}

// Dot products of up to 4 ring rows with x, lanes over chunks lane, lane + 32,
// ...: each x chunk is read once for all the rows.  nr is warp-uniform.
template <int DT>
__device__ __forceinline__ void rows4(const char *const (&rp)[4], int nr, int nv, int lane, const XView &x,
                                      float (&out)[4]) {
    constexpr int V = RowDot<DT>::VEC;
    float a[4][V];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int k = 0; k < V; ++k) a[r][k] = 0.f;
#pragma unroll 2
    for (int c = lane; c < nv; c += 32) {
        const float4 x0 = x.L(c), y0 = DT == MR_DTYPE_F32 ? float4{} : x.H(c);
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (r < nr) RowDot<DT>::add(a[r], ld_smem(reinterpret_cast<const uint4 *>(rp[r]) + c), x0, y0);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] = fold<DT>(a[r]);
}

// y[i] = row_i . x for i < n (n <= kRowBatch); rows start at `base` with
// stride row_bytes.  Many rows: one warp per row.  Few rows: several warps
// split each row and their partials are summed in a fixed order.  Ends with a
// compute barrier, after which every read of `base` has completed.
template <bool FROM_SMEM>
__device__ void rows_dot(const char *base, int dtype, int cols, int n, const XView &x, float *y, Control &c) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = static_cast<size_t>(cols) * esize(dtype);
    if (n >= kEngineWarps) {
        for (int i = warp; i < n; i += kEngineWarps) {
            float acc = row_partial_any<FROM_SMEM>(dtype, base + i * row_bytes, cols, lane, 32, lane, x);
            acc = warp_sum(acc);
            if (lane == 0) y[i] = acc;
        }
        csync();
        return;
    }
    const int wpr = kEngineWarps / n;
    const int i = warp / wpr, part = warp % wpr;
    if (i < n) {
        float acc = row_partial_any<FROM_SMEM>(dtype, base + i * row_bytes, cols, part * 32 + lane, 32 * wpr,
                                               part == 0 ? lane : -1, x);
        acc = warp_sum(acc);
        if (lane == 0) c.partial[i * wpr + part] = acc;
    }
    csync();
    if (threadIdx.x < n) {
        float total = 0.f;
        for (int p = 0; p < wpr; ++p) total += c.partial[threadIdx.x * wpr + p];
        y[threadIdx.x] = total;
    }
    csync();
}

// ---- GEMV phases ----------------------------------------------------------------------
struct Epi {
    unsigned long long best = 0;
    int nonfinite = 0;
};

// Loads a GEMV phase's input vector into `in` (no barrier): the token's
// embedding row (layer 0), else the previous phase's exchange words.  With
// `gain` (an RMSNorm input; NULL gain pointer = non-affine), stores x * gain
// instead and returns this thread's part of sum(x^2) in `ss`: the norm's
// factor is then applied to the dot products (kernels.cl:19-28 computes
// (x * scale) * gain; scale * (W . (x * gain)) differs by float32 rounding).
// Threads first .. first + count - 1 of the compute warps take part.
__device__ bool read_input(const GemvPhase &g, int cols, const StepInfo &info, int p, float *in, StepState *st,
                           bool norm, const void *gain, float &ss, int first, int count) {
    const int t = threadIdx.x - first;
    ss = 0.f;
    // the phase's raw input row, kept for the work between steps (aux_step.cuh): stored by
    // the CTA that owns row 0 of the first segment
    float *saved = nullptr;
    if (g.save_in) {
        int r0, r1;
        seg_cta_rows(g.seg[0], blockIdx.x, gridDim.x, g.skip, r0, r1);
        if (r0 == 0 && r1 > 0) saved = g.save_in + static_cast<size_t>(info.position % g.save_rows) * cols;
    }
    auto put = [&](int j, float v) {
        if (saved) saved[j] = v;
        if (norm) {
            ss = fmaf(v, v, ss);
            if (gain) v = __fmul_rn(v, load_weight(gain, g.norm_gain_dtype, j));
        }
        in[g.xsplit ? split_index(j, cols) : j] = v;
    };
    if (t < 0 || t >= count) return true;
    if (g.input_kind == IN_EMBED_ROW) {
        for (int j = t; j < cols; j += count)
            put(j, load_weight(g.embed, g.embed_dtype, static_cast<size_t>(info.token) * cols + j));
        return true;
    }
    const unsigned tag = info.tag_base + p - g.in_back;
    bool ok = true;
    for (int base = 0; base < cols && ok; base += 4 * count) {
        float v[4];
        ok = read_words(
            [&](int u) -> const Word * {
                const int e = base + u * count + t;
                return e < cols ? g.in + e : nullptr;
            },
            tag, v, st, p);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = base + u * count + t;
            if (ok && e < cols) put(e, v[u]);
        }
    }
    return ok;
}

// In-place RMSNorm of the input (kernels.cl:25-27: scale = 1/sqrt(mean + eps);
// y = (x * scale) * gain).  `gain` is in shared memory or global memory (or
// NULL: non-affine).  Ends with a compute barrier.
__device__ void norm_input(float *in, int cols, float eps, const void *gain, int gain_dtype, Control &c) {
    float ss = 0.f;
    for (int j = threadIdx.x; j < cols; j += kEngineThreads) ss = fmaf(in[j], in[j], ss);
    ss = block_sum(ss, c);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    for (int j = threadIdx.x; j < cols; j += kEngineThreads) {
        const float gn = gain ? load_weight(gain, gain_dtype, j) : 1.0f;
        in[j] = __fmul_rn(__fmul_rn(in[j], scale), gn);
    }
    csync();
}


// Finishes output row r of segment s (dot product `val`, RMSNorm factor
// already applied): exchange word, residual update, or logit.
__device__ __forceinline__ void finish_row(const GemvPhase &g, int s, int r, float val, const StepInfo &info, int p,
                                           Control &c, Epi &e) {
    const unsigned tag = info.tag_base + p;
    switch (g.epilogue) {
        case EPI_STORE: st_word_all(c, g.seg[s].out + r, val, tag); break;
        case EPI_RESIDUAL:  // model.py:282-283; x rows of this CTA live in shared memory
        case EPI_RESIDUAL_KEEP: {
            const float xn = __fadd_rn(c.xres[r - info.xr0], __fmul_rn(g.scale, val));
            c.xres[r - info.xr0] = xn;
            if (g.epilogue == EPI_RESIDUAL) st_word_all(c, g.x + r, xn, tag);
            break;
        }
        case EPI_LOGITS: {
            float *dst = g.logits + static_cast<size_t>(info.logits_row) * g.seg[0].rows + r;
            if (c.ranks == 1) *dst = val;
            else
                for (int j = 0; j < c.ranks; ++j) *peer_ptr(c, j, dst) = val;  // every rank holds all logits
            if (!isfinite(val)) e.nonfinite = 1;
            else e.best = max(e.best, argmax_key(val, r));
            break;
        }
        default: break;  // EPI_SWIGLU: see swiglu_row
    }
}
// kernels.cl:46-50: out = (g / (1 + exp(-g))) * u
__device__ __forceinline__ void swiglu_row(const GemvPhase &g, int r, float gt, float up, const StepInfo &info, int p,
                                           const Control &c) {
    st_word_all(c, g.out + r, __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up), info.tag_base + p);
}

__device__ void finish_logits(StepState *st, Control &c, Epi &e) {
    unsigned long long best = e.best;
    for (int offset = 16; offset > 0; offset >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, offset));
    const int nonfinite = __any_sync(0xffffffffu, e.nonfinite);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        c.best[warp] = best;
        if (nonfinite) atomicExch(&st->nonfinite, 1);
    }
    csync();
    if (threadIdx.x == 0) {
        unsigned long long m = 0;
        for (int w = 0; w < kEngineWarps; ++w) m = max(m, c.best[w]);
        if (m) atomicMax(&st->best, m);
    }
}

// ---- piece groups ----------------------------------------------------------------
// Piece of the group holding dot product v (v < t.rows).
__device__ __forceinline__ int find_piece(const GroupTable &t, int v) {
    int k = 0;
    while (t.p[k].seg < 0 || v >= t.p[k].vbase + t.p[k].n) ++k;
    return k;
}
// Row table of piece group t (pieces from stream index cbase), entries
// first, first + step, ...: .x = ring byte offset of dot product v's row,
// .y = segment << 30 | SwiGLU gate partner << 22 | output row (the partner of
// an up row is the index of the gate row of the same output, one piece back).
// Looked up once per group, off the path from the input to the dot products.
__device__ __forceinline__ void build_rows(const GemvPhase &g, const GroupTable &t, int cbase, const Control &c,
                                           int2 *rows, int first, int step) {
    for (int v = first; v < t.rows; v += step) {
        const int k = find_piece(t, v);
        const GroupPiece &pc = t.p[k];
        const int sgi = pc.seg, i = v - pc.vbase;
        const Segment &seg = g.seg[sgi];
        const int partner = (g.epilogue == EPI_SWIGLU && sgi == 1) ? v - pc.n : 0;
        rows[v] = make_int2(c.offset[(cbase + k) % kQueue] + i * seg.cols * esize(seg.dtype),
                            static_cast<int>((static_cast<unsigned>(sgi) << 30) | (static_cast<unsigned>(partner) << 22) |
                                             static_cast<unsigned>(pc.row0 + i)));
    }
}
__device__ __forceinline__ int row_seg(int2 r) { return static_cast<int>(static_cast<unsigned>(r.y) >> 30); }
__device__ __forceinline__ int row_partner(int2 r) { return static_cast<int>((static_cast<unsigned>(r.y) >> 22) & 255u); }
__device__ __forceinline__ int row_out(int2 r) { return static_cast<int>(static_cast<unsigned>(r.y) & 0x3FFFFFu); }

// y[v] = row_v . x for the group's rows, all of dtype DT.  Many rows: each
// warp takes its rows (v = warp + 15k) four at a time, reading each x chunk
// once for the four (shared memory bandwidth, not arithmetic, bounds this
// loop: x read per row would cost twice the weight bytes); few rows: several
// warps split each row and their partials are summed in a fixed order.  Ends with a compute barrier (none when the group has no rows).
template <int DT>
__device__ void group_dots_t(const GemvPhase &g, const GroupTable &t, const int2 *rows, const Smem &sm, const XView &x,
                             float *y) {
    Control &c = *sm.c;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = t.rows, cols = g.seg[0].cols, nv = cols / RowDot<DT>::VEC;
    if (R >= kEngineWarps) {
        for (int j0 = 0;; j0 += 4) {
            int nr = 0;
#pragma unroll
            for (int r = 0; r < 4; ++r)
                if (warp + kEngineWarps * (j0 + r) < R) nr = r + 1;
            if (nr == 0) break;  // warp-uniform
            const char *ring = reinterpret_cast<const char *>(sm.ring);
            const char *rp[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) rp[r] = ring + rows[warp + kEngineWarps * (r < nr ? j0 + r : j0)].x;
            float out[4];
            rows4<DT>(rp, nr, nv, lane, x, out);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (r < nr) {
                    const float sum = warp_sum(out[r]);
                    if (lane == 0) y[warp + kEngineWarps * (j0 + r)] = sum;
                }
            }
        }
        csync();
    } else if (R > 0) {
        const int P = kEngineWarps / R;
        const int v = warp / P, part = warp % P;
        if (v < R) {
            const char *row = reinterpret_cast<const char *>(sm.ring) + rows[v].x;
            float acc = row_partial<DT, true>(row, cols, part * 32 + lane, 32 * P, part == 0 ? lane : -1, x);
            acc = warp_sum(acc);
            if (lane == 0) {
                if (P == 1) y[v] = acc;  // one warp per row: its sum is the dot product
                else c.partial[v * P + part] = acc;
            }
        }
        csync();
        if (P > 1) {
            if (threadIdx.x < R) {
                float total = 0.f;
                for (int q = 0; q < P; ++q) total += c.partial[threadIdx.x * P + q];
                y[threadIdx.x] = total;
            }
            csync();
        }
    }
}

// Segments of different dtypes in one phase (plain x): one row at a time.
__device__ void group_dots_mixed(const GemvPhase &g, const GroupTable &t, const int2 *rows, const Smem &sm,
                                 const float *in, float *y) {
    Control &c = *sm.c;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = t.rows, cols = g.seg[0].cols;
    if (R >= kEngineWarps) {
        for (int v = warp; v < R; v += kEngineWarps) {
            const int dt = g.seg[row_seg(rows[v])].dtype;
            const char *row = reinterpret_cast<const char *>(sm.ring) + rows[v].x;
            const float a = warp_sum(row_partial_any<true>(dt, row, cols, lane, 32, lane, x_plain(in, dt)));
            if (lane == 0) y[v] = a;
        }
        csync();
    } else if (R > 0) {
        const int P = kEngineWarps / R;
        const int v = warp / P, part = warp % P;
        if (v < R) {
            const int dt = g.seg[row_seg(rows[v])].dtype;
            const char *row = reinterpret_cast<const char *>(sm.ring) + rows[v].x;
            float acc = row_partial_any<true>(dt, row, cols, part * 32 + lane, 32 * P, part == 0 ? lane : -1,
                                              x_plain(in, dt));
            acc = warp_sum(acc);
            if (lane == 0) c.partial[v * P + part] = acc;
        }
        csync();
        if (threadIdx.x < R) {
            float total = 0.f;
            for (int q = 0; q < P; ++q) total += c.partial[threadIdx.x * P + q];
            y[threadIdx.x] = total;
        }
        csync();
    }
}

__device__ void group_dots(const GemvPhase &g, const GroupTable &t, const int2 *rows, const Smem &sm, const float *in,
                           float *y) {
    const int cols = g.seg[0].cols;
    switch (g.wdtype) {
        case MR_DTYPE_BF16: group_dots_t<MR_DTYPE_BF16>(g, t, rows, sm, x_split(in, cols), y); break;
        case MR_DTYPE_F16: group_dots_t<MR_DTYPE_F16>(g, t, rows, sm, x_split(in, cols), y); break;
        case MR_DTYPE_F32: group_dots_t<MR_DTYPE_F32>(g, t, rows, sm, x_plain(in, MR_DTYPE_F32), y); break;
        default: group_dots_mixed(g, t, rows, sm, in, y); break;
    }
}

// Epilogue of the group: thread v finishes dot product v.  `scale` is the
// input's RMSNorm factor (applied here: scale * (W . (x * gain)) equals the
// reference's W . ((x * scale) * gain) up to float32 rounding).
__device__ void group_epilogue(const GemvPhase &g, const GroupTable &t, const int2 *rows, const float *y, float scale,
                               const StepInfo &info, int p, Control &c, Epi &e) {
    const int v = threadIdx.x;
    if (v >= t.rows) return;
    const int2 ri = rows[v];
    const int s = row_seg(ri), r = row_out(ri);
    const float val = g.norm ? __fmul_rn(y[v], scale) : y[v];
    if (g.epilogue != EPI_SWIGLU) {
        finish_row(g, s, r, val, info, p, c, e);
    } else if (s == 1) {  // the gate row of the same output is in the previous piece
        const float gy = y[row_partner(ri)];
        swiglu_row(g, r, g.norm ? __fmul_rn(gy, scale) : gy, val, info, p, c);
    }
}

// Record copies on an mbarrier: issued and awaited counts (thread 0), so that
// an early exit can wait for a copy still in flight.
// Warp 0 requests a record (`bytes`, a multiple of 16) into shared memory:
// 16 bytes per lane per pass with cp.async, which leaves the bulk-copy
// engine to the weight stream (a record queued behind weight pieces there
// would hold up the warp that leads every phase).  Complete once the issuing
// lanes have passed cp_async_wait_all.
__device__ __forceinline__ void warp_fetch(void *dst, const void *src, int bytes) {
    for (int o = (threadIdx.x & 31) * 16; o < bytes; o += 32 * 16)
        cp_async16_cg(static_cast<char *>(dst) + o, static_cast<const char *>(src) + o);
    cp_async_commit();
}

// GEMV whose weights stream through the shared-memory ring.  `cidx` is the
// index of the next piece of this CTA's stream (the same in every thread).
// The first group's table is already in shared memory.  A CTA without rows
// in the phase skips it (and reads none of its input).  The first group's
// pieces are awaited (warp 0) while the input words are polled; the RMSNorm's
// sum of squares is taken while the input is scaled by the gain, and its
// factor is applied in the epilogue.
__device__ bool gemv_bulk(const GemvPhase &g, int p, StepState *st, const StepInfo &info, const StepControl &ctl,
                          const Smem &sm, int &cidx, const Tracer &tr) {
    Control &c = *sm.c;
    GroupTable *tables = c.group[p & 1];
    if (tables[0].count == 0 && !tables[0].more) return true;  // no rows here
    const int cols = g.seg[0].cols;
    const bool tracing = tr.rec != nullptr;
    const GroupTable *src = ctl.groups + g.group_offset + static_cast<size_t>(blockIdx.x) * g.group_stride;
    float *in = sm.scratch;
    bool ok = true;
    if (threadIdx.x < 32 && tables[0].more) warp_fetch(&tables[1], src + 1, sizeof(GroupTable));  // one group ahead
    float ss = 0.f;
    if (threadIdx.x < 32) {
        // warp 0: the first group's pieces, then its row table, while warps 1.. bring in the input
        ok = wait_group(c, cidx, tables[0].count, st, p, tracing);
        if (ok) build_rows(g, tables[0], cidx, c, c.rowinfo[0], threadIdx.x, 32);
    } else {
        // the norm gain travels as the first group's first piece: every reading
        // thread observes its landing (long since, normally) before using it
        const void *gain = g.norm_gain;
        if (g.norm && tables[0].count > 0 && tables[0].p[0].seg < 0) {
            ok = wait_bar(&c.full[cidx % kQueue], (cidx / kQueue) & 1, st, c, p, false);
            gain = sm.ring + c.offset[cidx % kQueue];
        }
        ok = ok && read_input(g, cols, info, p, in, st, g.norm != 0, gain, ss, 32, kEngineThreads - 32);
    }
    if (g.norm) {
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) c.red[threadIdx.x >> 5] = ss;
    }
    if (!csync_and(ok)) {
        if (threadIdx.x == 0) c.abort = 1;
        return false;
    }
    tr.mark(0);
    float scale = 1.0f;
    if (g.norm) {
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kEngineWarps; ++w) total += c.red[w];
        // kernels.cl:25-27: scale = 1/sqrt(mean + eps)
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)cols), g.norm_eps)));
    }
    tr.mark(1);
    Epi e;
    for (int gi = 0;; ++gi) {
        const GroupTable &t = tables[gi & 1];
        const int2 *rows = c.rowinfo[gi & 1];
        float *y = c.y[gi & 1];
        group_dots(g, t, rows, sm, in, y);
        const int count = t.count;
        const bool more = t.more != 0;
        // the group's pieces are consumed: released by threads that finish no row (count <= 16, rows <= 256)
        const int rel = kEngineThreads - 1 - threadIdx.x;
        if (rel < count) mbar_arrive(&c.empty[(cidx + rel) % kQueue]);
        group_epilogue(g, t, rows, y, scale, info, p, c, e);
        cidx += count;
        if (!more) break;
        ok = true;
        if (threadIdx.x < 32) {
            cp_async_wait_all();  // table gi + 1
            __syncwarp();
            ok = wait_group(c, cidx, tables[(gi + 1) & 1].count, st, p, tracing);
            if (ok) build_rows(g, tables[(gi + 1) & 1], cidx, c, c.rowinfo[(gi + 1) & 1], threadIdx.x, 32);
        }
        if (!csync_and(ok)) {
            if (threadIdx.x == 0) c.abort = 1;
            return false;
        }
        // every thread has finished group gi's epilogue: its table buffer takes group gi + 2
        if (threadIdx.x < 32 && tables[(gi + 1) & 1].more) warp_fetch(&tables[gi & 1], src + gi + 2, sizeof(GroupTable));
    }
    tr.mark(2);
    tr.waits(c.wait_ns, c.late);
    if (g.epilogue == EPI_LOGITS) finish_logits(st, c, e);
    return true;
}

// GEMV reading weights straight from global memory (shapes the ring cannot
// take).  A CTA without rows in the phase skips it.
__device__ bool gemv_direct(const GemvPhase &g, int p, StepState *st, const StepInfo &info, const Smem &sm) {
    Control &c = *sm.c;
    const int G = gridDim.x, b = blockIdx.x, cols = g.seg[0].cols;
    bool mine = false;
    for (int s = 0; s < g.nseg; ++s) {
        int r0, r1;
        seg_cta_rows(g.seg[s], b, G, g.skip, r0, r1);
        mine = mine || r1 > r0;
    }
    if (!mine) return true;
    float *in = sm.scratch;
    float ss;
    const bool ok = read_input(g, cols, info, p, in, st, false, nullptr, ss, 0, kEngineThreads);
    if (!csync_and(ok)) {
        if (threadIdx.x == 0) c.abort = 1;
        return false;
    }
    if (g.norm) norm_input(in, cols, g.norm_eps, g.norm_gain, g.norm_gain_dtype, c);
    Epi e;
    int buf = 0;
    const bool paired = g.epilogue == EPI_SWIGLU;
    for (int s = 0; s < (paired ? 1 : g.nseg); ++s) {
        int r0, r1;
        seg_cta_rows(g.seg[s], b, G, g.skip, r0, r1);
        for (int rb = r0; rb < r1; rb += kRowBatch) {
            const int n = min(kRowBatch, r1 - rb);
            for (int part = 0; part < (paired ? 2 : 1); ++part) {
                const Segment &seg = g.seg[s + part];
                const char *base = static_cast<const char *>(seg.w) + static_cast<size_t>(rb) * cols * esize(seg.dtype);
                rows_dot<false>(base, seg.dtype, cols, n, x_plain(in, seg.dtype), c.y[buf], c);
                // the gate and up rows of index i are finished by the same thread
                for (int i = threadIdx.x; i < n; i += kEngineThreads) {
                    if (!paired) finish_row(g, s, rb + i, c.y[buf][i], info, p, c, e);
                    else if (part == 0) c.gate[i] = c.y[buf][i];
                    else swiglu_row(g, rb + i, c.gate[i], c.y[buf][i], info, p, c);
                }
                buf ^= 1;
            }
        }
    }
    if (g.epilogue == EPI_LOGITS) finish_logits(st, c, e);
    return true;
}

// ---- grouped-query attention ------------------------------------------------------
// In-place per-head RMSNorm (optional) + RoPE of a [dim] vector held by one warp
// in shared memory (kernels.cl rms 19-28 then rope 30-44).  `gain` is in
// shared memory (float) or NULL; cos / sin of position * inv_freq[p] come
// from the launch's table (the same float32 values the reference computes).
__device__ void norm_rope_warp(float *v, int dim, const float *gain, float eps, bool do_norm,
                               const float *rope_cos, const float *rope_sin, int split_half) {
    const int lane = threadIdx.x & 31;
    if (do_norm) {
        float ss = 0.f;
        for (int j = lane; j < dim; j += 32) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
        for (int j = lane; j < dim; j += 32) v[j] = __fmul_rn(__fmul_rn(v[j], scale), gain ? gain[j] : 1.0f);
        __syncwarp();
    }
    const int half = dim / 2;
    for (int p = lane; p < half; p += 32) {
        const int j = split_half ? p : 2 * p, k = split_half ? p + half : 2 * p + 1;
        const float u = v[j], w = v[k], cs = rope_cos[p], sn = rope_sin[p];
        v[j] = __fsub_rn(__fmul_rn(u, cs), __fmul_rn(w, sn));
        v[k] = __fadd_rn(__fmul_rn(u, sn), __fmul_rn(w, cs));
    }
    __syncwarp();
}

// Issues the asynchronous loads of one key/value tile (logical keys tb ..
// tb+nt-1 of KV head g) into kt / vt.  Ring rows were written by earlier
// launches (the newest row, written in this launch, is patched from shared
// memory by its owner), relay rows by the host.
__device__ void issue_tile(const AttnPhase &a, int g, int tb, int nt, int start, int length, const AttnLayout &L,
                           float *kt, float *vt) {
    const int d = a.dim, cap = a.capacity;
    auto row_src = [&](int lt, const float *&kr, const float *&vr) {
        if (lt < length) {
            const size_t row = static_cast<size_t>(g) * cap + (start + lt) % cap;
            kr = a.k_cache + row * d;
            vr = a.v_cache + row * d;
        } else {
            const size_t row = static_cast<size_t>(g) * a.relay_capacity + (lt - length);
            kr = a.relay_k + row * d;
            vr = a.relay_v + row * d;
        }
    };
    if ((d & 3) == 0) {
        const int per_row = d / 4;
        for (int e = threadIdx.x; e < nt * per_row; e += kEngineThreads) {
            const int t = e / per_row, j = (e - t * per_row) * 4;
            const float *kr, *vr;
            row_src(tb + t, kr, vr);
            cp_async16_cg(kt + t * L.kstride + j, kr + j);
            cp_async16_cg(vt + t * L.vstride + j, vr + j);
        }
    } else {
        for (int e = threadIdx.x; e < nt * d; e += kEngineThreads) {
            const int t = e / d, j = e - t * d;
            const float *kr, *vr;
            row_src(tb + t, kr, vr);
            cp_async4(kt + t * L.kstride + j, kr + j);
            cp_async4(vt + t * L.vstride + j, vr + j);
        }
    }
    cp_async_commit();
}

// Attention work geometry of this step for one layer.
struct AttnGeometry {
    int count, length, start, total, chunks, chunk_len;
    __device__ AttnGeometry(const AttnPhase &a, const StepInfo &info) {
        count = info.position + 1;
        length = min(count, a.capacity);
        start = (count - length) % a.capacity;
        total = length + (a.relay_count ? __ldcg(a.relay_count) : 0);
        chunks = attn_chunks(total, a.kv_n, gridDim.x);
        chunk_len = (total + chunks - 1) / chunks;
    }
};

// Requests the first key/value tile of this CTA's first attention unit (all
// compute threads; completed by the attention phase's first wait).  Called at
// the end of the preceding phase: ring rows come from earlier launches (the
// newest row, written in this launch, is patched from shared memory by its
// owner), relay rows from the host.
__device__ bool attn_first_tile(const AttnPhase &a, const StepInfo &info, const Smem &sm) {
    const AttnGeometry geo(a, info);
    const int unit = blockIdx.x;
    if (unit >= a.kv_n * geo.chunks) return false;
    const int g = a.kv_lo + unit / geo.chunks, c = unit % geo.chunks;
    const int t0 = c * geo.chunk_len, t1 = min(geo.total, t0 + geo.chunk_len);
    if (t0 >= t1) return false;
    const AttnLayout L = attn_layout(a.heads / a.kv_heads, a.dim);
    issue_tile(a, g, t0, min(kKeyTile, t1 - t0), geo.start, geo.length, L, sm.attn + L.kt, sm.attn + L.vt);
    return true;
}

// Reads n exchange words carrying `tag`, word q at addr(q), into dst[q]
// (shared memory), four per thread per pass; every compute thread takes part
// (no barrier).
template <typename Addr>
__device__ bool read_to_smem(int n, Addr addr, unsigned tag, float *dst, StepState *st, int phase) {
    bool ok = true;
    for (int base = 0; base < n && ok; base += 4 * kEngineThreads) {
        float v[4];
        ok = read_words(
            [&](int u) -> const Word * {
                const int q = base + u * kEngineThreads + threadIdx.x;
                return q < n ? addr(q) : nullptr;
            },
            tag, v, st, phase);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int q = base + u * kEngineThreads + threadIdx.x;
            if (ok && q < n) dst[q] = v[u];
        }
    }
    return ok;
}

// After publishing its own chunk, every unit of a KV head merges one slice
// (1/chunks) of the head group's attention output: the reference's softmax
// over all keys (model.py:95-116) equals sum_c w_c acc_c with
// w_c = exp(m_c - M) / sum_c' exp(m_c' - M) l_c', M the largest chunk maximum.
// The slice's accumulators of every chunk and every (head, chunk) maximum and
// sum are brought into shared memory (`scratch`, spread over all threads:
// one polling round), the weights are formed per (head, chunk), and the
// output rows go out as exchange words for the o projection.
__device__ bool merge_slice(const AttnPhase &a, int g, int gq, int chunks, int c, float *scratch, unsigned tag,
                            StepState *st, int phase, const Control &ctl) {
    const int d = a.dim, stride = d + 2, n = gq * d;
    const int per = (n + chunks - 1) / chunks, e0 = c * per, e1 = min(n, e0 + per);
    const int nacc = max(0, e1 - e0) * chunks, npair = gq * chunks;
    auto rec = [&](int i, int cc) {
        return a.partial + (static_cast<size_t>(g * gq + i) * kMaxAttnChunks + cc) * stride;
    };
    float *vals = scratch, *ml = scratch + nacc, *wgt = ml + 2 * npair;
    // vals[k * chunks + cc] = acc of element e0 + k in chunk cc; ml[2 * (i * chunks + cc) + {0, 1}] = max, sum
    const bool ok = read_to_smem(
        nacc + 2 * npair,
        [&](int q) -> const Word * {
            if (q < nacc) {
                const int k = q / chunks, cc = q - k * chunks, e = e0 + k;
                return rec(e / d, cc) + (e % d);
            }
            const int r = (q - nacc) >> 1, i = r / chunks, cc = r - i * chunks;
            return rec(i, cc) + d + ((q - nacc) & 1);
        },
        tag, vals, st, phase);
    if (!csync_and(ok)) return false;
    for (int r = threadIdx.x; r < npair; r += kEngineThreads) {
        const int i = r / chunks, cc = r - i * chunks;
        const float *mi = ml + 2 * i * chunks;
        float mx = -INFINITY;
        for (int u = 0; u < chunks; ++u) mx = fmaxf(mx, mi[2 * u]);
        float den = 0.f;
        for (int u = 0; u < chunks; ++u) {
            const float mu = mi[2 * u];
            den += (mu == -INFINITY) ? 0.f : expf(mu - mx) * mi[2 * u + 1];
        }
        const float m = mi[2 * cc];
        wgt[r] = (m == -INFINITY) ? 0.f : expf(m - mx) / den;
    }
    csync();
    for (int k = threadIdx.x; k < e1 - e0; k += kEngineThreads) {
        const int e = e0 + k, i = e / d;
        float sum = 0.f;
        for (int cc = 0; cc < chunks; ++cc) sum = fmaf(wgt[i * chunks + cc], vals[k * chunks + cc], sum);
        st_word_all(ctl, a.out + static_cast<size_t>(g * gq) * d + e, sum, tag);
    }
    return true;
}

// Scores of one key tile with per-warp softmax statistics: element
// e = i * kKeyTile + t (query head i, key t), so every warp holds 32 keys of
// one head; p[e] = exp(score - warp max), the warp's max and sum go to
// wm / wl[e / 32].  Keys t >= nt (and any past the tile) contribute nothing.
// D: the head dim at compile time (unrolled), 0: at run time.
template <int D>
__device__ __forceinline__ void tile_scores(const float *q, const float *kt, int kstride, int d, int gq, int nt,
                                            float sqrt_d, float *p, float *wm, float *wl) {
    const int lane = threadIdx.x & 31;
    const int dim = D ? D : d;
    for (int e = threadIdx.x; e < gq * kKeyTile; e += kEngineThreads) {
        const int i = e / kKeyTile, t = e - i * kKeyTile;
        const bool live = t < nt;
        const float *qi = q + i * dim, *kr = kt + (live ? t : 0) * kstride;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        if (D || (dim & 3) == 0) {
#pragma unroll 8
            for (int j = 0; j < dim; j += 4) {
                const float4 qa = *reinterpret_cast<const float4 *>(qi + j);
                const float4 ka = *reinterpret_cast<const float4 *>(kr + j);
                s0 = fmaf(qa.x, ka.x, s0);
                s1 = fmaf(qa.y, ka.y, s1);
                s2 = fmaf(qa.z, ka.z, s2);
                s3 = fmaf(qa.w, ka.w, s3);
            }
        } else {
            for (int j = 0; j < dim; ++j) s0 = fmaf(qi[j], kr[j], s0);
        }
        const float sc = live ? __fdiv_rn((s0 + s1) + (s2 + s3), sqrt_d) : -INFINITY;  // kernels.cl:72
        const float mw = warp_max(sc);
        const float pr = (live && mw != -INFINITY) ? expf(sc - mw) : 0.f;
        const float lw = warp_sum(pr);
        p[e] = pr;
        if (lane == 0) {
            wm[e >> 5] = mw;
            wl[e >> 5] = lw;
        }
    }
}

// Value mix of one key tile into the running (acc, max m, sum l) of
// model.py:95-116's softmax: the two warp halves of head i are brought to the
// common maximum.  m / l are read from buffer `par` and written to par ^ 1
// (every thread reads the old state of its head).
template <int D>
__device__ __forceinline__ void tile_mix(const float *p, const float *vt, int vstride, int d, int gq, int nt,
                                         const float *wm, const float *wl, float *acc, float *mrow, float *lrow,
                                         int par) {
    const int dim = D ? D : d;
    for (int e = threadIdx.x; e < gq * dim; e += kEngineThreads) {
        const int i = e / dim, j = e - i * dim;
        const float m_old = mrow[par * gq + i], m0 = wm[2 * i], m1 = wm[2 * i + 1];
        const float mx = fmaxf(m_old, fmaxf(m0, m1));
        const float cf = (m_old == -INFINITY) ? 0.f : expf(m_old - mx);
        const float f0 = (m0 == -INFINITY) ? 0.f : expf(m0 - mx);
        const float f1 = (m1 == -INFINITY) ? 0.f : expf(m1 - mx);
        const float *pi = p + i * kKeyTile;
        float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
        if (nt == kKeyTile) {
#pragma unroll
            for (int t = 0; t < 32; t += 2) {
                a0 = fmaf(pi[t], vt[t * vstride + j], a0);
                a1 = fmaf(pi[t + 1], vt[(t + 1) * vstride + j], a1);
                b0 = fmaf(pi[32 + t], vt[(32 + t) * vstride + j], b0);
                b1 = fmaf(pi[33 + t], vt[(33 + t) * vstride + j], b1);
            }
        } else {  // rows past nt hold stale data: never read them
            for (int t = 0; t < min(nt, 32); ++t) a0 = fmaf(pi[t], vt[t * vstride + j], a0);
            for (int t = 32; t < nt; ++t) b0 = fmaf(pi[t], vt[t * vstride + j], b0);
        }
        acc[e] = fmaf(f1, b0 + b1, fmaf(f0, a0 + a1, acc[e] * cf));
        if (j == 0) {
            mrow[(par ^ 1) * gq + i] = mx;
            lrow[(par ^ 1) * gq + i] = fmaf(f1, wl[2 * i + 1], fmaf(f0, wl[2 * i], lrow[par * gq + i] * cf));
        }
    }
}

// Work unit = (KV head g, chunk c of the attended rows): one pass over the
// chunk's keys (in tiles of kKeyTile) for the group's query heads.  The
// group's raw q rows and (owner) this token's raw k/v rows come from the qkv
// phase as exchange words; the newest row (this token's key and value,
// appended to the ring by the unit that owns it) is patched into its tile in
// shared memory.  Every unit publishes its chunk (acc, max, sum) as exchange
// words and then merges one slice of the group's output (merge_slice).  With
// chunks >= 2 there are never more units than CTAs, so a merging unit never
// waits for work queued behind it on its own CTA.
template <int D>
__device__ bool attn_gqa_phase_t(const AttnPhase &a, const StepInfo &info, int ph, const Smem &sm,
                                 bool first_tile_issued, StepState *st, const Tracer &tr) {
    const int G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = a.dim, gq = a.heads / a.kv_heads;
    const AttnGeometry geo(a, info);
    const int count = geo.count, cap = a.capacity, length = geo.length, start = geo.start, total = geo.total;
    const int chunks = geo.chunks, chunk_len = geo.chunk_len;
    const float sqrt_d = __fsqrt_rn(static_cast<float>(d));  // divisor, kernels.cl:72
    const int stride = d + 2;
    const unsigned in_tag = info.tag_base + ph - 1, out_tag = info.tag_base + ph;
    const unsigned q_tag = info.tag_base + ph - a.q_back;

    const AttnLayout L = attn_layout(gq, d);
    float *q = sm.attn + L.q, *knew = sm.attn + L.knew, *vnew = sm.attn + L.vnew;
    float *kt = sm.attn + L.kt, *vt = sm.attn + L.vt, *p = sm.attn + L.p, *acc = sm.attn + L.acc;
    float *mrow = sm.attn + L.m, *lrow = sm.attn + L.l, *wm = sm.attn + L.wm, *wl = wm + 2 * gq;
    float *gains = sm.c->gains;

    for (int unit = blockIdx.x; unit < a.kv_n * chunks; unit += G) {
        const int g = a.kv_lo + unit / chunks, c = unit % chunks;
        const int t0 = c * chunk_len, t1 = min(total, t0 + chunk_len);
        const int newest = length - 1;
        const bool owner = newest >= t0 && newest < t1;
        // 1. the first tile (unless requested at the end of the previous phase), norm gains
        if (t0 < t1 && !(first_tile_issued && unit == static_cast<int>(blockIdx.x)))
            issue_tile(a, g, t0, min(kKeyTile, t1 - t0), start, length, L, kt, vt);
        if (a.qk_norm && a.q_gain)
            for (int e = threadIdx.x; e < 2 * d; e += kEngineThreads)
                gains[e] = load_weight(e < d ? a.q_gain : a.k_gain, a.gain_dtype, e < d ? e : e - d);
        for (int e = threadIdx.x; e < gq * d; e += kEngineThreads) acc[e] = 0.f;
        if (threadIdx.x < gq) {
            mrow[threadIdx.x] = -INFINITY;
            lrow[threadIdx.x] = 0.f;
        }
        int par = 0;  // the running max / sum are in buffer par
        // 2. the group's q rows and (owner) this token's k / v rows
        bool ok = true;
        const int nq = gq * d, nread = nq + (owner ? 2 * d : 0);
        for (int base = 0; base < nread && ok; base += 4 * kEngineThreads) {
            float v[4];
            ok = read_words_tagged(
                [&](int u) -> const Word * {
                    const int e = base + u * kEngineThreads + threadIdx.x;
                    return e >= nread ? nullptr
                           : e < nq   ? a.q_raw + static_cast<size_t>(g) * nq + e
                           : e < nq + d ? a.k_raw + static_cast<size_t>(g) * d + (e - nq)
                                        : a.v_raw + static_cast<size_t>(g) * d + (e - nq - d);
                },
                [&](int u) { return base + u * kEngineThreads + static_cast<int>(threadIdx.x) < nq ? q_tag : in_tag; },
                v, st, ph);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = base + u * kEngineThreads + threadIdx.x;
                if (!ok || e >= nread) continue;
                if (e < nq) q[e] = v[u];
                else if (e < nq + d) knew[e - nq] = v[u];
                else vnew[e - nq - d] = v[u];
            }
        }
        bool first = true;
        for (int tb = t0; tb < t1; tb += kKeyTile) {
            const int nt = min(kKeyTile, t1 - tb);
            cp_async_wait_all();
            if (!csync_and(ok)) return false;
            if (first) {
                tr.mark(0);
                // 3. query heads: RMSNorm + RoPE; the owner also finishes this token's key/value
                const float *qg = (a.qk_norm && a.q_gain) ? gains : nullptr;
                const float *kg = (a.qk_norm && a.k_gain) ? gains + d : nullptr;
                const float *rc = sm.c->rope_cos, *rs = sm.c->rope_sin;
                for (int i = warp; i < gq; i += kEngineWarps)
                    norm_rope_warp(q + i * d, d, qg, a.norm_eps, a.qk_norm != 0, rc, rs, a.split_half);
                if (owner && warp == kEngineWarps - 1) {
                    norm_rope_warp(knew, d, kg, a.norm_eps, a.qk_norm != 0, rc, rs, a.split_half);
                    const size_t slot = static_cast<size_t>(g) * cap + (count - 1) % cap;
                    for (int j = lane; j < d; j += 32) a.k_cache[slot * d + j] = knew[j];
                }
                if (owner && warp == kEngineWarps - 2) {
                    const size_t slot = static_cast<size_t>(g) * cap + (count - 1) % cap;
                    for (int j = lane; j < d; j += 32) a.v_cache[slot * d + j] = vnew[j];
                }
                csync();
                first = false;
                tr.mark(1);
            }
            if (owner && newest >= tb && newest < tb + nt) {
                // the tile holds the ring's previous occupant of the newest slot: patch it
                const int t = newest - tb;
                for (int j = threadIdx.x; j < d; j += kEngineThreads) {
                    kt[t * L.kstride + j] = knew[j];
                    vt[t * L.vstride + j] = vnew[j];
                }
                csync();
            }
            // 4. scores, with the softmax statistics of each warp's 32 keys
            tile_scores<D>(q, kt, L.kstride, d, gq, nt, sqrt_d, p, wm, wl);
            csync();
            // 5. value mix and the running softmax state
            tile_mix<D>(p, vt, L.vstride, d, gq, nt, wm, wl, acc, mrow, lrow, par);
            par ^= 1;
            csync();
            if (tb + kKeyTile < t1) issue_tile(a, g, tb + kKeyTile, min(kKeyTile, t1 - tb - kKeyTile), start, length, L, kt, vt);
        }
        tr.mark(2);
        // 7. the chunk's result: output rows (single chunk), else publish the chunk and merge a slice
        if (chunks == 1) {
            for (int e = threadIdx.x; e < gq * d; e += kEngineThreads) {
                const int i = e / d, j = e - i * d;
                st_word_all(*sm.c, a.out + static_cast<size_t>(g * gq + i) * d + j, __fdiv_rn(acc[e], lrow[par * gq + i]),
                            out_tag);
            }
        } else {
            for (int e = threadIdx.x; e < gq * d; e += kEngineThreads) {
                const int i = e / d, j = e - i * d;
                st_word(a.partial + (static_cast<size_t>(g * gq + i) * kMaxAttnChunks + c) * stride + j, acc[e], out_tag);
            }
            if (threadIdx.x < gq) {
                Word *rec = a.partial + (static_cast<size_t>(g * gq + threadIdx.x) * kMaxAttnChunks + c) * stride;
                st_word(rec + d, mrow[par * gq + threadIdx.x], out_tag);
                st_word(rec + d + 1, lrow[par * gq + threadIdx.x], out_tag);
            }
            if (!merge_slice(a, g, gq, chunks, c, kt, out_tag, st, ph, *sm.c)) return false;  // the tiles are free
        }
        csync();
    }
    return true;
}

__device__ bool attn_gqa_phase(const AttnPhase &a, const StepInfo &info, int ph, const Smem &sm,
                               bool first_tile_issued, StepState *st, const Tracer &tr) {
    switch (a.dim) {
        case 64: return attn_gqa_phase_t<64>(a, info, ph, sm, first_tile_issued, st, tr);
        case 128: return attn_gqa_phase_t<128>(a, info, ph, sm, first_tile_issued, st, tr);
        default: return attn_gqa_phase_t<0>(a, info, ph, sm, first_tile_issued, st, tr);
    }
}

}  // namespace

__global__ void __launch_bounds__(kBlockThreads, 1)
    decode_step_kernel(const Phase *__restrict__ phases, int nphases, StepState *st, StepControl ctl) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem sm;
    sm.c = reinterpret_cast<Control *>(smem_raw);
    sm.scratch = reinterpret_cast<float *>(smem_raw + ((sizeof(Control) + 127) & ~size_t(127)));
    sm.ring = reinterpret_cast<unsigned char *>(sm.scratch) +
              ((static_cast<size_t>(ctl.scratch_floats) * 4 + 127) & ~size_t(127));
    sm.ring_bytes = ctl.ring_bytes;
    sm.attn = sm.scratch + ctl.attn_base;
    Control &c = *sm.c;
    const int head_phase = nphases - 2;  // the phase list ends with the head, then the step end
    __shared__ StepInfo info;
    __shared__ unsigned long long base;
    __shared__ int skip, need_head;
    if (threadIdx.x == 0) {
        volatile StepState *vs = st;
        skip = vs->stopped || vs->error;
        const int pos = vs->position;
        const int rel = pos - ctl.feed_base;
        info.position = pos;
        info.token = (rel >= 0 && rel < ctl.feed_len) ? ctl.feed[rel] : vs->token;
        // split over ranks, every step ends with the argmax exchange: no rank starts the next
        // step (and overwrites exchange words in the others' arenas) before all have finished
        need_head = ctl.return_all || rel >= ctl.feed_len - 1 || ctl.ranks > 1;
        info.logits_row = ctl.return_all ? rel % ctl.logits_rows : 0;
        info.tag_base = ctl.tag_base;
        cta_row_range(ctl.xres_n, blockIdx.x, gridDim.x, ctl.xres_skip, info.xr0, info.xr1);
        info.xr0 += ctl.xres_lo;
        info.xr1 += ctl.xres_lo;
        base = vs->barrier_base;
        if (!skip && pos >= ctl.context_length) {
            if (blockIdx.x == 0) atomicCAS(&st->error, 0, 3);
            skip = 1;
        }
        if (!skip && (info.token < 0 || info.token >= ctl.vocab_size)) {
            if (blockIdx.x == 0) atomicCAS(&st->error, 0, 4);
            skip = 1;
        }
        if (!skip) {
            for (int i = 0; i < kQueue; ++i) {
                mbar_init(&c.full[i], 1);
                mbar_init(&c.empty[i], 1);
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            c.abort = 0;
            c.wait_ns = 0;
            c.late = 0;
            c.ranks = ctl.ranks;
            c.withhold = ctl.withhold_phase >= 0;
            c.withhold_tag = ctl.tag_base + static_cast<unsigned>(ctl.withhold_phase);
            c.arena = ctl.arena;
            for (int j = 0; j < kMaxRanks; ++j) c.peers[j] = ctl.peers[j];
        }
        if (!skip && ctl.trace && blockIdx.x == 0) ctl.trace[0] = global_ns();
    }
    __syncthreads();  // the last block-wide barrier: the producer warp leaves below
    if (skip) return;
    if (threadIdx.x >= kEngineThreads) {  // the producer warp
        if (threadIdx.x == kEngineThreads) produce(ctl, need_head != 0, head_phase, st, sm);
        return;
    }
    // RoPE cos / sin of this launch's position (kernels.cl:30-44 computes them per element)
    for (int i = threadIdx.x; i < ctl.rope_pairs; i += kEngineThreads) {
        const float angle = __fmul_rn(static_cast<float>(info.position), ctl.inv_freq[i]);
        c.rope_cos[i] = cosf(angle);
        c.rope_sin[i] = sinf(angle);
    }
    // this CTA's rows of the residual stream start as the token's embedding
    for (int i = threadIdx.x; i < info.xr1 - info.xr0; i += kEngineThreads)
        c.xres[i] = load_weight(ctl.embed, ctl.embed_dtype, static_cast<size_t>(info.token) * ctl.hidden + info.xr0 + i);
    // the first phase's records: descriptor, then its first group table (two round trips, once per launch)
    bool ok = true;
    if (threadIdx.x < 32) {
        warp_fetch(&c.phase[0], &phases[0], sizeof(Phase));
        cp_async_wait_all();
        __syncwarp();
        if (c.phase[0].kind == PH_GEMV && c.phase[0].gemv.bulk) {
            warp_fetch(&c.group[0][0],
                       ctl.groups + c.phase[0].gemv.group_offset +
                           static_cast<size_t>(blockIdx.x) * c.phase[0].gemv.group_stride,
                       sizeof(GroupTable));
            cp_async_wait_all();
        }
    }
    ok = csync_and(ok);
    int cidx = 0, executed = 0;
    bool tile_issued = false;  // the next attention phase's first tile is in flight
    for (int p = 0; p < nphases - 1 && ok; ++p) {
        const Phase &ph = c.phase[p & 1];
        if (ph.layer < 0 && !need_head) break;  // the head is the last phase before the step end
        const bool prefetch = p + 1 < nphases - 1;
        if (threadIdx.x < 32 && prefetch) {  // the next phase's descriptor and first group table
            warp_fetch(&c.phase[(p + 1) & 1], &phases[p + 1], sizeof(Phase));
            if (ph.next_groups >= 0)
                warp_fetch(&c.group[(p + 1) & 1][0],
                           ctl.groups + ph.next_groups + static_cast<size_t>(blockIdx.x) * ph.next_group_stride,
                           sizeof(GroupTable));
        }
        const Tracer tr{ctl.trace ? ctl.trace + 1 + static_cast<size_t>(executed) * (gridDim.x * kTraceStamps + 1)
                                  : nullptr};
        if (ph.kind == PH_GEMV) {
            if (ph.gemv.bulk) ok = gemv_bulk(ph.gemv, p, st, info, ctl, sm, cidx, tr);
            else ok = gemv_direct(ph.gemv, p, st, info, sm);
        } else if (ph.kind == PH_ATTN_GQA) {
            ok = attn_gqa_phase(ph.attn, info, p, sm, tile_issued, st, tr);
            tile_issued = false;
        }
        if (!ok) break;
        // the next phase's records have landed (normally long since); the barrier publishes them
        cp_async_wait_all();
        ok = csync_and(ok);
        if (!ok) break;
        // an attention phase next: its first key/value tile loads while the q/k/v words are awaited
        if (prefetch && c.phase[(p + 1) & 1].kind == PH_ATTN_GQA)
            tile_issued = attn_first_tile(c.phase[(p + 1) & 1].attn, info, sm);
        tr.mark(3);
        if (tr.rec && blockIdx.x == 0 && threadIdx.x == 0) tr.rec[gridDim.x * kTraceStamps] = global_ns();
        ++executed;
    }
    cp_async_wait_all();
    // one grid barrier per step: every CTA's logits and argmax are in before the step ends
    int barriers = 0;
    if (c.ranks > 1 && need_head) __threadfence_system();  // this thread's logits in every rank's arena
    if (ok && need_head) {
        ++barriers;
        ok = grid_barrier(st, base + static_cast<unsigned long long>(barriers) * gridDim.x, nphases - 2, c, [] {});
    }
    if (!ok) {  // every copy this CTA requested has landed (cp_async_wait_all above)
        if (threadIdx.x == 0) c.abort = 1;
        return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        volatile StepState *s = st;
        const int pos = info.position;
        const int rel = pos - ctl.feed_base;
        if (need_head) {
            unsigned long long key = s->best;
            if (c.ranks > 1) {
                // every rank's argmax of its vocabulary rows (and its non-finite flag) to every
                // rank; then the greatest (ties: the lowest index, as numpy.argmax)
                const unsigned tag = info.tag_base + nphases;  // no phase of this launch uses it
                Word *mine = ctl.best_slots + 4 * ctl.rank;
                const unsigned parts[3] = {static_cast<unsigned>(key >> 32), static_cast<unsigned>(key),
                                           static_cast<unsigned>(s->nonfinite)};
                __threadfence_system();
                for (int j = 0; j < c.ranks; ++j)
                    for (int q = 0; q < 3; ++q)
                        st_word_sys(peer_ptr(c, j, mine + q), (static_cast<Word>(tag) << 32) | parts[q]);
                const uint64_t start = global_ns();
                for (int j = 0; j < c.ranks; ++j) {
                    Word w[3];
                    for (int q = 0; q < 3; ++q) {
                        for (;;) {
                            w[q] = ld_word(ctl.best_slots + 4 * j + q);
                            if (word_ok(w[q], tag)) break;
                            if (global_ns() - start > wait_limit(st)) {
                                atomicCAS(&st->error, 0, 1000 + nphases);
                                break;
                            }
                        }
                    }
                    const unsigned long long kj = (static_cast<unsigned long long>(static_cast<unsigned>(w[0])) << 32) |
                                                  static_cast<unsigned>(w[1]);
                    key = max(key, kj);
                    if (static_cast<unsigned>(w[2])) s->nonfinite = 1;
                }
                __threadfence_system();  // the logits every rank stored here are in before the step ends
            }
            const int arg = key ? argmax_index(key) : -1;
            s->last_argmax = arg;
            s->best = 0ull;
            if (ctl.gen_max > 0 && rel >= ctl.feed_len - 1) {
                if (s->nonfinite) {
                    s->stopped = 1;
                } else {
                    const int n = s->gen_count;
                    if (ctl.gen_out) ctl.gen_out[n] = arg;
                    s->gen_count = n + 1;
                    s->token = arg;
                    if (arg == ctl.eos || n + 1 >= ctl.gen_max) s->stopped = 1;
                }
            }
        }
        s->position = pos + 1;
        s->barrier_base = base + static_cast<unsigned long long>(barriers) * gridDim.x;
        __threadfence();
    }
}

size_t decode_control_bytes() { return (sizeof(Control) + 127) & ~size_t(127); }

}  // namespace mr
