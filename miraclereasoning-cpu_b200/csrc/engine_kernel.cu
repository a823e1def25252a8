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
// Weight streaming (see engine.cuh): thread 0 is the producer of a
// shared-memory byte ring fed by TMA bulk copies (cp.async.bulk, completion
// on one mbarrier per piece); every thread consumes pieces in the same order.
// All waits are bounded (2 s): a wait that gives up records an error code in
// StepState, every CTA drains its in-flight copies (bounded) and returns, and
// the host raises.
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
constexpr int kMaxMergeHeads = 64;

// Fixed part of the dynamic shared memory; the scratch floats and the weight
// ring follow it.
struct Control {
    unsigned long long mbar[kQueue];
    int offset[kQueue];
    float partial[kEngineWarps * kEngineWarps];
    float y[2][kRowBatch];   // y[0]: rows of the current piece; y[1]: gate rows (SwiGLU)
    float red[kEngineWarps];
    float merge_w[kMaxMergeHeads * kMaxAttnChunks];
    unsigned long long best[kEngineWarps];
    int flag, ok;
    // producer state (written by thread 0 only)
    int issued, consumed, head_offset;
};

struct StepInfo {
    int position, token, logits_row;
};

// Phase trace checkpoints (no-ops unless the launch carries a trace buffer).
struct Tracer {
    unsigned long long *rec;  // this phase's record, or NULL
    __device__ void mark(int i) const {
        if (!rec) return;
        __syncthreads();
        if (threadIdx.x == 0) rec[blockIdx.x * kTraceStamps + i] = global_ns();
    }
};

struct Smem {
    Control *c;
    float *scratch;
    unsigned char *ring;
    int ring_bytes;
};

__device__ __forceinline__ void row_range(int rows, int b, int g, int &r0, int &r1) {
    r0 = static_cast<int>(static_cast<long long>(rows) * b / g);
    r1 = static_cast<int>(static_cast<long long>(rows) * (b + 1) / g);
}

__device__ __forceinline__ int esize(int dtype) { return dtype == MR_DTYPE_F32 ? 4 : 2; }
__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

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
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}
// Copy n floats produced in this launch into shared memory: 16-byte .cg
// granules when both ends are 16-byte aligned and n % 4 == 0, else loads
// batched in registers (no store-to-load ordering between iterations).
__device__ void copy_fresh(float *dst, const float *src, int n) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 && (n & 3) == 0) {
        for (int e = threadIdx.x * 4; e < n; e += blockDim.x * 4) cp_async16_cg(dst + e, src + e);
        cp_async_wait_all();
        return;
    }
    for (int base = 0; base < n; base += 4 * blockDim.x) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = base + u * blockDim.x + threadIdx.x;
            v[u] = e < n ? __ldcg(src + e) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = base + u * blockDim.x + threadIdx.x;
            if (e < n) dst[e] = v[u];
        }
    }
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
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, unsigned long long *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ---- piece stream (host-precomputed table, see PieceDesc) ---------------------------
__device__ __forceinline__ const PieceDesc *cta_pieces(const StepControl &ctl) {
    return ctl.pieces + static_cast<size_t>(blockIdx.x) * ctl.piece_stride;
}

// Producer (thread 0): issue the next pieces of this CTA's stream while the
// ring and the mbarrier queue have room.  Pieces of the head phase are only
// streamed when this step computes logits.
__device__ void refill(const StepControl &ctl, bool need_head, int head_phase, const Smem &sm) {
    Control &c = *sm.c;
    const PieceDesc *table = cta_pieces(ctl);
    const int count = ctl.piece_count[blockIdx.x];
    bool fenced = false;
    while (c.issued < count && c.issued - c.consumed < kQueue) {
        const PieceDesc d = table[c.issued];
        if (!need_head && d.phase == head_phase) return;
        const int bytes = static_cast<int>(d.bytes);
        int off;
        if (c.issued == c.consumed) {
            off = 0;
        } else {
            const int head = c.head_offset, tail = c.offset[c.consumed % kQueue];
            if (head == tail) return;  // full
            if (head > tail) {
                if (head + bytes <= sm.ring_bytes) off = head;
                else if (bytes <= tail) off = 0;
                else return;
            } else {
                if (head + bytes <= tail) off = head;
                else return;
            }
        }
        if (!fenced) {
            // the region may have been read through the generic proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fenced = true;
        }
        const int slot = c.issued % kQueue;
        c.offset[slot] = off;
        bulk_load(sm.ring + off, d.src, d.bytes, &c.mbar[slot]);
        c.head_offset = off + bytes;
        ++c.issued;
    }
}

// Bounded wait for piece `idx` (all threads).
__device__ bool wait_piece(const Smem &sm, int idx, StepState *st, int phase) {
    unsigned long long *bar = &sm.c->mbar[idx % kQueue];
    const int parity = (idx / kQueue) & 1;
    uint64_t start = 0;
    for (unsigned spin = 0;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 255u) == 255u) {
            if (*reinterpret_cast<volatile int *>(&st->error)) return false;
            const uint64_t now = global_ns();
            if (!start) {
                start = now;
            } else if (now - start > kWaitLimitNs) {
                atomicCAS(&st->error, 0, 1000 + phase);
                return false;
            }
        }
    }
}

// Thread 0, on exit: wait (bounded) for every issued copy so that no bulk copy
// writes into shared memory after the CTA has left.
__device__ void drain(const Smem &sm) {
    Control &c = *sm.c;
    const uint64_t start = global_ns();
    for (int idx = c.consumed; idx < c.issued; ++idx) {
        while (!mbar_try_wait(&c.mbar[idx % kQueue], (idx / kQueue) & 1)) {
            if (global_ns() - start > kWaitLimitNs) return;
        }
    }
}

// ---- grid barrier ------------------------------------------------------------------
// Release-add arrival (cumulative over the CTA's writes ordered by bar.sync),
// acquire polling by thread 0, bounded by kWaitLimitNs.
__device__ bool grid_barrier(StepState *st, unsigned long long target, int phase, const Smem &sm) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(&st->barrier) : "memory");
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
                } else if (now - start > kWaitLimitNs) {
                    atomicCAS(&st->error, 0, 1000 + phase);
                    ok = 0;
                    break;
                }
            }
        }
        sm.c->ok = ok;
    }
    __syncthreads();
    return sm.c->ok != 0;
}

// Deterministic block sum (same order in every CTA -> identical bits).
__device__ float block_sum(float v, Control &c) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) c.red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float total = lane < kEngineWarps ? c.red[lane] : 0.f;
        total = warp_sum(total);
        if (lane == 0) c.red[0] = total;
    }
    __syncthreads();
    const float total = c.red[0];
    __syncthreads();
    return total;
}

// ---- dot products -------------------------------------------------------------------
template <int DT>
struct RowDot;

template <>
struct RowDot<MR_DTYPE_BF16> {
    static constexpr int VEC = 8;
    __device__ static float chunk(const uint4 &w, const float *x) {
        const float4 a = *reinterpret_cast<const float4 *>(x), b = *reinterpret_cast<const float4 *>(x + 4);
        float acc = __uint_as_float(w.x << 16) * a.x;
        acc = fmaf(__uint_as_float(w.x & 0xffff0000u), a.y, acc);
        acc = fmaf(__uint_as_float(w.y << 16), a.z, acc);
        acc = fmaf(__uint_as_float(w.y & 0xffff0000u), a.w, acc);
        acc = fmaf(__uint_as_float(w.z << 16), b.x, acc);
        acc = fmaf(__uint_as_float(w.z & 0xffff0000u), b.y, acc);
        acc = fmaf(__uint_as_float(w.w << 16), b.z, acc);
        acc = fmaf(__uint_as_float(w.w & 0xffff0000u), b.w, acc);
        return acc;
    }
};

template <>
struct RowDot<MR_DTYPE_F16> {
    static constexpr int VEC = 8;
    __device__ static float chunk(const uint4 &w, const float *x) {
        const float4 a = *reinterpret_cast<const float4 *>(x), b = *reinterpret_cast<const float4 *>(x + 4);
        const __half2 *h = reinterpret_cast<const __half2 *>(&w);
        const float2 p0 = __half22float2(h[0]), p1 = __half22float2(h[1]), p2 = __half22float2(h[2]),
                     p3 = __half22float2(h[3]);
        float acc = p0.x * a.x;
        acc = fmaf(p0.y, a.y, acc);
        acc = fmaf(p1.x, a.z, acc);
        acc = fmaf(p1.y, a.w, acc);
        acc = fmaf(p2.x, b.x, acc);
        acc = fmaf(p2.y, b.y, acc);
        acc = fmaf(p3.x, b.z, acc);
        acc = fmaf(p3.y, b.w, acc);
        return acc;
    }
};

template <>
struct RowDot<MR_DTYPE_F32> {
    static constexpr int VEC = 4;
    __device__ static float chunk(const uint4 &w, const float *x) {
        const float4 a = *reinterpret_cast<const float4 *>(x);
        float acc = __uint_as_float(w.x) * a.x;
        acc = fmaf(__uint_as_float(w.y), a.y, acc);
        acc = fmaf(__uint_as_float(w.z), a.z, acc);
        acc = fmaf(__uint_as_float(w.w), a.w, acc);
        return acc;
    }
};

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
// byte length is not a multiple of 16 use scalar loads only.
template <int DT, bool FROM_SMEM>
__device__ float row_partial(const char *rp, int cols, int first, int stride, int tail_lane, const float *x) {
    using D = RowDot<DT>;
    const int nv = cols / D::VEC;
    const size_t row_bytes = static_cast<size_t>(cols) * esize(DT);
    float acc = 0.f;
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
            acc += D::chunk(w0, x + c * D::VEC);
            acc += D::chunk(w1, x + (c + stride) * D::VEC);
            acc += D::chunk(w2, x + (c + 2 * stride) * D::VEC);
            acc += D::chunk(w3, x + (c + 3 * stride) * D::VEC);
        }
        for (; c < nv; c += stride) acc += D::chunk(FROM_SMEM ? ld_smem(v + c) : ld_stream(v + c), x + c * D::VEC);
        if (!FROM_SMEM && tail_lane >= 0)
            for (int j = nv * D::VEC + tail_lane; j < cols; j += 32) acc = fmaf(load_weight(rp, DT, j), x[j], acc);
    } else if (tail_lane >= 0) {
        for (int j = tail_lane; j < cols; j += 32) acc = fmaf(load_weight(rp, DT, j), x[j], acc);
    }
    return acc;
}

template <bool FROM_SMEM>
__device__ float row_partial_any(int dtype, const char *rp, int cols, int first, int stride, int tail_lane,
                                 const float *x) {
    switch (dtype) {
        case MR_DTYPE_BF16: return row_partial<MR_DTYPE_BF16, FROM_SMEM>(rp, cols, first, stride, tail_lane, x);
        case MR_DTYPE_F16: return row_partial<MR_DTYPE_F16, FROM_SMEM>(rp, cols, first, stride, tail_lane, x);
        default: return row_partial<MR_DTYPE_F32, FROM_SMEM>(rp, cols, first, stride, tail_lane, x);
    }
}

// y[i] = row_i . x for i < n (n <= kRowBatch) into c.y[0]; rows start at `base`
// with stride row_bytes.  Many rows: one warp per row.  Few rows: several
// warps split each row and their partials are summed in a fixed order.
template <bool FROM_SMEM>
__device__ void rows_dot(const char *base, int dtype, int cols, int n, const float *x, Control &c) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = static_cast<size_t>(cols) * esize(dtype);
    if (n >= kEngineWarps) {
        for (int i = warp; i < n; i += kEngineWarps) {
            float acc = row_partial_any<FROM_SMEM>(dtype, base + i * row_bytes, cols, lane, 32, lane, x);
            acc = warp_sum(acc);
            if (lane == 0) c.y[0][i] = acc;
        }
        __syncthreads();
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
    __syncthreads();
    if (threadIdx.x < n) {
        float total = 0.f;
        for (int p = 0; p < wpr; ++p) total += c.partial[threadIdx.x * wpr + p];
        c.y[0][threadIdx.x] = total;
    }
    __syncthreads();
}

// ---- GEMV phases ----------------------------------------------------------------------
__device__ void merge_attention(const AttnMerge &m, int position, float *in, Control &c) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = min(position + 1, m.capacity) + (m.relay_count ? __ldcg(m.relay_count) : 0);
    const int chunks = attn_chunks(total, m.kv_heads, gridDim.x);
    const int stride = m.dim + 2;
    for (int h = warp; h < m.heads; h += kEngineWarps) {
        const float *base = m.partial + static_cast<size_t>(h) * kMaxAttnChunks * stride;
        const float mc = lane < chunks ? __ldcg(base + lane * stride + m.dim) : -INFINITY;
        const float lc = lane < chunks ? __ldcg(base + lane * stride + m.dim + 1) : 0.f;
        const float mx = warp_max(mc);
        const float w = (mc == -INFINITY) ? 0.f : expf(mc - mx);
        const float den = warp_sum(w * lc);
        if (lane < kMaxAttnChunks) c.merge_w[h * kMaxAttnChunks + lane] = lane < chunks ? w / den : 0.f;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < m.heads * m.dim; e += blockDim.x) {
        const int h = e / m.dim, j = e % m.dim;
        const float *base = m.partial + static_cast<size_t>(h) * kMaxAttnChunks * stride + j;
        float v[kMaxAttnChunks];
#pragma unroll
        for (int cc = 0; cc < kMaxAttnChunks; ++cc) v[cc] = cc < chunks ? __ldcg(base + cc * stride) : 0.f;
        const float *w = c.merge_w + h * kMaxAttnChunks;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int cc = 0; cc < kMaxAttnChunks; cc += 2) {
            a0 = fmaf(w[cc], v[cc], a0);
            a1 = fmaf(w[cc + 1], v[cc + 1], a1);
        }
        in[e] = a0 + a1;
    }
    __syncthreads();
}

__device__ void load_input(const GemvPhase &g, int cols, const StepInfo &info, float *in, Control &c) {
    if (g.input_kind == IN_EMBED_ROW) {
        for (int j = threadIdx.x; j < cols; j += blockDim.x) {
            const float v = load_weight(g.embed, g.embed_dtype, static_cast<size_t>(info.token) * cols + j);
            in[j] = v;
            if (g.embed_copy && blockIdx.x == 0) g.embed_copy[j] = v;
        }
        __syncthreads();
    } else if (g.input_kind == IN_ATTN_MERGE) {
        merge_attention(g.merge, info.position, in, c);
    } else {
        copy_fresh(in, g.in, cols);
        __syncthreads();
    }
}

struct Epi {
    unsigned long long best = 0;
    int nonfinite = 0;
};

// Epilogue of rows [row0, row0+n) of segment `s` whose dot products are in c.y[0].
__device__ void epilogue(const GemvPhase &g, int s, int row0, int n, const StepInfo &info, Control &c, Epi &e) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = row0 + i;
        const float y = c.y[0][i];
        switch (g.epilogue) {
            case EPI_STORE: g.seg[s].out[r] = y; break;
            case EPI_RESIDUAL: g.x[r] = __fadd_rn(__ldcg(g.x + r), __fmul_rn(g.scale, y)); break;
            case EPI_SWIGLU:
                if (s == 0) {
                    c.y[1][i] = y;
                } else {
                    const float gt = c.y[1][i];
                    g.out[r] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), y);
                }
                break;
            case EPI_LOGITS:
                g.out[static_cast<size_t>(info.logits_row) * g.seg[0].rows + r] = y;
                if (!isfinite(y)) e.nonfinite = 1;
                else e.best = max(e.best, argmax_key(y, r));
                break;
        }
    }
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
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0;
        for (int w = 0; w < kEngineWarps; ++w) m = max(m, c.best[w]);
        if (m) atomicMax(&st->best, m);
    }
    __syncthreads();
}

// GEMV whose weights stream through the shared-memory ring.  `cidx` is the
// index of the next piece of this CTA's stream (the same in every thread).
__device__ bool gemv_bulk(const GemvPhase &g, int p, const StepControl &ctl, bool need_head, int head_phase,
                          StepState *st, const StepInfo &info, const Smem &sm, int &cidx, const Tracer &tr) {
    Control &c = *sm.c;
    const int cols = g.seg[0].cols;
    const PieceDesc *table = cta_pieces(ctl);
    const int count = ctl.piece_count[blockIdx.x];
    float *in = sm.scratch;
    auto consumed = [&]() {
        __syncthreads();
        if (threadIdx.x == 0) {
            ++c.consumed;
            refill(ctl, need_head, head_phase, sm);
        }
        ++cidx;
    };
    load_input(g, cols, info, in, c);
    tr.mark(0);
    if (g.norm) {
        float ss = 0.f;
        for (int j = threadIdx.x; j < cols; j += blockDim.x) ss = fmaf(in[j], in[j], ss);
        ss = block_sum(ss, c);
        // kernels.cl:25-27: scale = 1/sqrt(mean + eps); y = (x * scale) * gain
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), g.norm_eps)));
        const unsigned char *gain_smem = nullptr;
        if (g.gain_piece) {
            // every thread agrees on the outcome before any of them moves on
            if (!__syncthreads_and(wait_piece(sm, cidx, st, p))) return false;
            gain_smem = sm.ring + c.offset[cidx % kQueue];
        }
        for (int j = threadIdx.x; j < cols; j += blockDim.x) {
            float gain = 1.0f;
            if (gain_smem) gain = load_weight(gain_smem, g.norm_gain_dtype, j);
            else if (g.norm_gain) gain = load_weight(g.norm_gain, g.norm_gain_dtype, j);
            in[j] = __fmul_rn(__fmul_rn(in[j], scale), gain);
        }
        if (g.gain_piece) consumed();
        else __syncthreads();
    }
    tr.mark(1);
    Epi e;
    while (cidx < count) {
        const PieceDesc d = table[cidx];
        if (d.phase != p) break;
        if (!__syncthreads_and(wait_piece(sm, cidx, st, p))) return false;
        const Segment &s = g.seg[d.seg];
        const char *rows = reinterpret_cast<const char *>(sm.ring + c.offset[cidx % kQueue]);
        rows_dot<true>(rows, s.dtype, cols, d.nrows, in, c);
        epilogue(g, d.seg, d.row0, d.nrows, info, c, e);
        consumed();
    }
    tr.mark(2);
    if (g.epilogue == EPI_LOGITS) finish_logits(st, c, e);
    return true;
}

// GEMV reading weights straight from global memory (shapes the ring cannot take).
__device__ void gemv_direct(const GemvPhase &g, StepState *st, const StepInfo &info, const Smem &sm) {
    Control &c = *sm.c;
    const int G = gridDim.x, b = blockIdx.x, cols = g.seg[0].cols;
    float *in = sm.scratch;
    load_input(g, cols, info, in, c);
    if (g.norm) {
        float ss = 0.f;
        for (int j = threadIdx.x; j < cols; j += blockDim.x) ss = fmaf(in[j], in[j], ss);
        ss = block_sum(ss, c);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), g.norm_eps)));
        for (int j = threadIdx.x; j < cols; j += blockDim.x) {
            const float gain = g.norm_gain ? load_weight(g.norm_gain, g.norm_gain_dtype, j) : 1.0f;
            in[j] = __fmul_rn(__fmul_rn(in[j], scale), gain);
        }
        __syncthreads();
    }
    Epi e;
    const bool paired = g.epilogue == EPI_SWIGLU;
    for (int s = 0; s < (paired ? 1 : g.nseg); ++s) {
        int r0, r1;
        row_range(g.seg[s].rows, b, G, r0, r1);
        for (int rb = r0; rb < r1; rb += kRowBatch) {
            const int n = min(kRowBatch, r1 - rb);
            for (int part = 0; part < (paired ? 2 : 1); ++part) {
                const Segment &seg = g.seg[s + part];
                const char *base = static_cast<const char *>(seg.w) + static_cast<size_t>(rb) * cols * esize(seg.dtype);
                rows_dot<false>(base, seg.dtype, cols, n, in, c);
                epilogue(g, s + part, rb, n, info, c, e);
                __syncthreads();
            }
        }
    }
    if (g.epilogue == EPI_LOGITS) finish_logits(st, c, e);
}

// ---- grouped-query attention ------------------------------------------------------
__device__ __forceinline__ void rope_pair(float &u, float &v, float angle) {
    const float c = cosf(angle), s = sinf(angle);
    const float a = __fsub_rn(__fmul_rn(u, c), __fmul_rn(v, s));
    const float b = __fadd_rn(__fmul_rn(u, s), __fmul_rn(v, c));
    u = a;
    v = b;
}

// In-place per-head RMSNorm (optional) + RoPE of a [dim] vector held by one warp
// in shared memory (kernels.cl rms 19-28 then rope 30-44).  `gain` is in
// shared memory (float) or NULL.
__device__ void norm_rope_warp(float *v, int dim, const float *gain, float eps, bool do_norm,
                               const float *inv_freq, float position, int split_half) {
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
        float u = v[j], w = v[k];
        rope_pair(u, w, __fmul_rn(position, inv_freq[p]));
        v[j] = u;
        v[k] = w;
    }
    __syncwarp();
}

// Work unit = (KV head g, chunk c of the attended rows): one pass over the
// chunk's keys (in tiles of kKeyTile) for the group's query heads; writes the
// chunk's (acc, max, sum) for the consumer to merge.  All of a tile's global
// reads are issued at once with cp.async; the newest row (this token's key and
// value, appended to the ring by the unit that owns it) is patched into the
// tile in shared memory.
__device__ void attn_gqa_phase(const AttnPhase &a, const StepInfo &info, const Smem &sm, const Tracer &tr) {
    const int G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = a.dim, gq = a.heads / a.kv_heads;
    const int count = info.position + 1;
    const int cap = a.capacity;
    const int length = min(count, cap);
    const int start = (count - length) % cap;
    const int extra = a.relay_count ? __ldcg(a.relay_count) : 0;
    const int total = length + extra;
    const int chunks = attn_chunks(total, a.kv_heads, G);
    const int chunk_len = (total + chunks - 1) / chunks;
    const float pos_f = static_cast<float>(info.position);
    const float sqrt_d = __fsqrt_rn(static_cast<float>(d));  // divisor, kernels.cl:72
    const int stride = d + 2;

    // q and knew first: 16-byte cp.async targets (scratch is 128-byte aligned,
    // gq*d is a multiple of 4 whenever d is)
    float *q = sm.scratch;                             // [gq][d]
    float *knew = q + gq * d;                          // [d]
    float *kt = knew + d;                              // [kKeyTile][d+1]
    float *vt = kt + kKeyTile * (d + 1);               // [kKeyTile][d]
    float *p = vt + kKeyTile * d;                      // [gq][kKeyTile]
    float *acc = p + gq * kKeyTile;                    // [gq][d]
    float *mrow = acc + gq * d;                        // [gq]
    float *lrow = mrow + gq;                           // [gq]
    float *corr = lrow + gq;                           // [gq]
    float *gains = sm.c->y[1];                         // q gain [d], k gain [d] (kRowBatch >= 2 * 128)

    for (int unit = blockIdx.x; unit < a.kv_heads * chunks; unit += G) {
        const int g = unit / chunks, c = unit % chunks;
        const int t0 = c * chunk_len, t1 = min(total, t0 + chunk_len);
        const int newest = length - 1;
        const bool owner = newest >= t0 && newest < t1;
        // 1. issue: the group's raw q rows, the first key/value tile, and (owner) the raw k/v row
        if ((d & 3) == 0) {
            for (int e = threadIdx.x * 4; e < gq * d; e += blockDim.x * 4)
                cp_async16_cg(q + e, a.q_raw + static_cast<size_t>(g) * gq * d + e);
            if (owner)
                for (int e = threadIdx.x * 4; e < d; e += blockDim.x * 4)
                    cp_async16_cg(knew + e, a.k_raw + static_cast<size_t>(g) * d + e);
        } else {
            for (int e = threadIdx.x; e < gq * d; e += blockDim.x) q[e] = __ldcg(a.q_raw + static_cast<size_t>(g) * gq * d + e);
            if (owner)
                for (int e = threadIdx.x; e < d; e += blockDim.x) knew[e] = __ldcg(a.k_raw + static_cast<size_t>(g) * d + e);
        }
        if (a.qk_norm && a.q_gain)
            for (int e = threadIdx.x; e < 2 * d; e += blockDim.x)
                gains[e] = load_weight(e < d ? a.q_gain : a.k_gain, a.gain_dtype, e < d ? e : e - d);
        for (int e = threadIdx.x; e < gq * d; e += blockDim.x) acc[e] = 0.f;
        if (threadIdx.x < gq) {
            mrow[threadIdx.x] = -INFINITY;
            lrow[threadIdx.x] = 0.f;
        }
        bool first = true;
        for (int tb = t0; tb < t1; tb += kKeyTile) {
            const int nt = min(kKeyTile, t1 - tb);
            for (int e = threadIdx.x; e < nt * d; e += blockDim.x) {
                const int t = e / d, j = e % d, lt = tb + t;
                const float *kr, *vr;
                if (lt < length) {
                    const size_t row = static_cast<size_t>(g) * cap + (start + lt) % cap;
                    kr = a.k_cache + row * d;
                    vr = a.v_cache + row * d;
                } else {
                    const size_t row = static_cast<size_t>(g) * a.relay_capacity + (lt - length);
                    kr = a.relay_k + row * d;
                    vr = a.relay_v + row * d;
                }
                cp_async4(kt + t * (d + 1) + j, kr + j);
                cp_async4(vt + t * d + j, vr + j);
            }
            cp_async_wait_all();
            __syncthreads();
            if (first) tr.mark(0);
            if (first) {
                // 2. query heads: RMSNorm + RoPE; the owner also finishes this token's key/value
                const float *qg = (a.qk_norm && a.q_gain) ? gains : nullptr;
                const float *kg = (a.qk_norm && a.k_gain) ? gains + d : nullptr;
                for (int i = warp; i < gq; i += kEngineWarps)
                    norm_rope_warp(q + i * d, d, qg, a.norm_eps, a.qk_norm != 0, a.inv_freq, pos_f, a.split_half);
                if (owner && warp == kEngineWarps - 1) {
                    norm_rope_warp(knew, d, kg, a.norm_eps, a.qk_norm != 0, a.inv_freq, pos_f, a.split_half);
                    const size_t slot = static_cast<size_t>(g) * cap + (count - 1) % cap;
                    for (int j = lane; j < d; j += 32) a.k_cache[slot * d + j] = knew[j];
                }
                if (owner && warp == kEngineWarps - 2) {
                    const size_t slot = static_cast<size_t>(g) * cap + (count - 1) % cap;
                    for (int j = lane; j < d; j += 32) a.v_cache[slot * d + j] = __ldcg(a.v_raw + static_cast<size_t>(g) * d + j);
                }
                __syncthreads();
                first = false;
                tr.mark(1);
            }
            if (owner && newest >= tb && newest < tb + nt) {
                // the tile holds the ring's previous occupant of the newest slot: patch it
                const int t = newest - tb;
                for (int j = threadIdx.x; j < d; j += blockDim.x) {
                    kt[t * (d + 1) + j] = knew[j];
                    vt[t * d + j] = __ldcg(a.v_raw + static_cast<size_t>(g) * d + j);
                }
                __syncthreads();
            }
            // 3. scores (4 independent partial sums per dot product)
            for (int e = threadIdx.x; e < gq * nt; e += blockDim.x) {
                const int i = e / nt, t = e % nt;
                const float *qi = q + i * d, *kr = kt + t * (d + 1);
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
                int j = 0;
                for (; j + 3 < d; j += 4) {
                    s0 = fmaf(qi[j], kr[j], s0);
                    s1 = fmaf(qi[j + 1], kr[j + 1], s1);
                    s2 = fmaf(qi[j + 2], kr[j + 2], s2);
                    s3 = fmaf(qi[j + 3], kr[j + 3], s3);
                }
                for (; j < d; ++j) s0 = fmaf(qi[j], kr[j], s0);
                p[i * kKeyTile + t] = __fdiv_rn((s0 + s1) + (s2 + s3), sqrt_d);
            }
            __syncthreads();
            // 4. online softmax per query head
            for (int i = warp; i < gq; i += kEngineWarps) {
                float mt = -INFINITY;
                for (int t = lane; t < nt; t += 32) mt = fmaxf(mt, p[i * kKeyTile + t]);
                mt = warp_max(mt);
                const float m_old = mrow[i], m_new = fmaxf(m_old, mt);
                float sum = 0.f;
                for (int t = lane; t < nt; t += 32) {
                    const float e = (m_new == -INFINITY) ? 0.f : expf(p[i * kKeyTile + t] - m_new);
                    p[i * kKeyTile + t] = e;
                    sum += e;
                }
                sum = warp_sum(sum);
                if (lane == 0) {
                    const float cf = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                    corr[i] = cf;
                    lrow[i] = lrow[i] * cf + sum;
                    mrow[i] = m_new;
                }
            }
            __syncthreads();
            // 5. value mix (4 independent partial sums)
            for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
                const int i = e / d, j = e % d;
                const float *pi = p + i * kKeyTile;
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                int t = 0;
                for (; t + 3 < nt; t += 4) {
                    a0 = fmaf(pi[t], vt[t * d + j], a0);
                    a1 = fmaf(pi[t + 1], vt[(t + 1) * d + j], a1);
                    a2 = fmaf(pi[t + 2], vt[(t + 2) * d + j], a2);
                    a3 = fmaf(pi[t + 3], vt[(t + 3) * d + j], a3);
                }
                for (; t < nt; ++t) a0 = fmaf(pi[t], vt[t * d + j], a0);
                acc[e] = fmaf(acc[e], corr[i], (a0 + a1) + (a2 + a3));
            }
            __syncthreads();
        }
        tr.mark(2);
        // 6. publish the chunk partial: acc[d], running max, running sum
        for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
            const int i = e / d, j = e % d;
            a.partial[(static_cast<size_t>(g * gq + i) * kMaxAttnChunks + c) * stride + j] = acc[e];
        }
        if (threadIdx.x < gq) {
            float *rec = a.partial + (static_cast<size_t>(g * gq + threadIdx.x) * kMaxAttnChunks + c) * stride;
            rec[d] = mrow[threadIdx.x];
            rec[d + 1] = lrow[threadIdx.x];
        }
        __syncthreads();
    }
}

}  // namespace

__global__ void __launch_bounds__(kEngineThreads, 1)
    decode_step_kernel(const Phase *__restrict__ phases, int nphases, StepState *st, StepControl ctl) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem sm;
    sm.c = reinterpret_cast<Control *>(smem_raw);
    sm.scratch = reinterpret_cast<float *>(smem_raw + ((sizeof(Control) + 127) & ~size_t(127)));
    sm.ring = reinterpret_cast<unsigned char *>(sm.scratch) +
              ((static_cast<size_t>(ctl.scratch_floats) * 4 + 127) & ~size_t(127));
    sm.ring_bytes = ctl.ring_bytes;
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
        need_head = ctl.return_all || rel >= ctl.feed_len - 1;
        info.logits_row = ctl.return_all ? rel % ctl.logits_rows : 0;
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
            for (int i = 0; i < kQueue; ++i) mbar_init(&c.mbar[i], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            c.issued = c.consumed = c.head_offset = 0;
        }
    }
    __syncthreads();
    if (skip) return;
    if (threadIdx.x == 0) {
        if (ctl.trace && blockIdx.x == 0) ctl.trace[0] = global_ns();
        refill(ctl, need_head != 0, head_phase, sm);
    }
    __syncthreads();
    int barriers = 0, cidx = 0;
    bool ok = true;
    for (int p = 0; p < nphases && ok; ++p) {
        const Phase &ph = phases[p];
        if (ph.kind == PH_STEP_END) break;
        if (ph.layer < 0 && !need_head) continue;
        const Tracer tr{ctl.trace ? ctl.trace + 1 + static_cast<size_t>(barriers) * (gridDim.x * kTraceStamps + 1)
                                  : nullptr};
        if (ph.kind == PH_GEMV) {
            if (ph.gemv.bulk) ok = gemv_bulk(ph.gemv, p, ctl, need_head != 0, head_phase, st, info, sm, cidx, tr);
            else gemv_direct(ph.gemv, st, info, sm);
        } else if (ph.kind == PH_ATTN_GQA) {
            attn_gqa_phase(ph.attn, info, sm, tr);
        }
        if (!ok) break;
        tr.mark(3);
        ++barriers;
        ok = grid_barrier(st, base + static_cast<unsigned long long>(barriers) * gridDim.x, p, sm);
        if (ok && tr.rec && blockIdx.x == 0 && threadIdx.x == 0) tr.rec[gridDim.x * kTraceStamps] = global_ns();
    }
    __syncthreads();
    if (threadIdx.x == 0) drain(sm);  // nothing is in flight on the normal path; bounded either way
    if (!ok) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        volatile StepState *s = st;
        const int pos = info.position;
        const int rel = pos - ctl.feed_base;
        if (need_head) {
            const unsigned long long key = s->best;
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
