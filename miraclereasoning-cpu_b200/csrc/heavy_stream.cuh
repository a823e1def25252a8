// Heavy Medium weight streaming (included by heavy.cu only).
//
// k_stream: y = W x for the projections that carry the bytes of a token step
// (q | latent, o, the experts' gate | up and down, the head).  One CTA per
// SM; every CTA owns the same row slice [rows*c/G, rows*(c+1)/G) of every
// matrix ("segment") of the launch, so an expert launch is balanced whatever
// the routing chose, and the down projection's CTA owns output rows of every
// expert, which lets it apply the rank-order combine (model.py:251-255) in
// its epilogue instead of a separate kernel.
//
// Warp 8 (one elected lane) streams the CTA's rows into a shared-memory ring
// of 16 KB slots with cp.async.bulk (one "full" mbarrier per slot, completed
// by the copy's byte count); consumer warps 0-7 take the pieces round robin,
// compute their rows' dot products against the staged input and release the
// slot through its "empty" mbarrier.  Before a consumer waits on piece n's
// "full" barrier it waits for the producer's count of issued pieces to pass n:
// a parity wait can only tell a barrier's current phase from the one before
// it, and once piece n is issued the slot's previous phase (piece n - S) has
// completed, so the wait is never two phases ahead (which would return at once,
// before the copy landed).  Segments whose weights do not depend on
// the previous kernel (shared experts, every static projection) are streamed
// before griddepcontrol.wait, so their loads overlap the previous kernel's
// tail (the ring is sized so that the next kernel's CTAs fit on the SM beside
// this one's); routed experts follow once the routing is visible.
//
// Arithmetic per row: the same float32 products as k_gemv / k_expert_* (the
// fallback for rows that are not whole 16-byte chunks), summed in another order
// (rows_dot: lane l keeps one running sum per column of its chunks l, l + 32,
// ..., folded pairwise, then a warp sum), which keeps the FMAs independent; the
// input's RMSNorm is staged by 256 threads exactly as stage_input does.
#pragma once

namespace stream {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kSlotBytes = 16384;  // the largest piece
constexpr int kMaxSlots = 16;
constexpr int kMaxSegs = 12;
constexpr int kMaxPieceRows = 4;
constexpr int kMaxPeers = 8;

enum Mode { kPlain = 0, kSwiglu = 1, kDown = 2 };

struct Seg {
    const void *w;   // [rows, cols] in the launch's dtype
    const void *w2;  // kSwiglu: the up matrix (w = gate)
    float *y;        // kPlain: output rows
    int rows;
    int slot;        // kSwiglu / kDown: the expert slot (routed 0..max_k-1 in rank order, shared after)
};

struct Args {
    int mode, dtype, cols, slots;  // slots: ring slots of slot_bytes
    int slot_bytes;                // one piece (<= kSlotBytes), a multiple of 128
    Seg seg[kMaxSegs];
    int nseg;                      // static segments (streamed before the dependency wait)
    // routed experts (kSwiglu / kDown): slots 0..active-1 = expert chosen[k]
    const void *const *dyn_w, *const *dyn_w2;
    const int *chosen, *active;
    int max_k, dyn_rows, experts;  // experts: the routed ids' range (a routing outside it is an error)
    // input: kPlain / kSwiglu one vector (RMSNorm(x, gain) when norm); kDown every slot's act row
    const float *x;
    int norm, gain_dtype;
    const void *gain;
    float eps;
    const float *acts;             // kDown: [max_k + shared][cols]
    int shared;
    // outputs
    float *act_out;                // kSwiglu: [max_k + shared][rows]
    int residual;                  // kPlain: y = y + scale * (W x)
    float scale;
    const float *weights;          // kDown: routed weights [max_k]
    float shared_scale;            // kDown: residual_scale / S
    float *xres;                   // kDown: x += scale * combine
    // expert parallel (ranks > 1): only this rank's experts (id % ranks == rank) are streamed,
    // and kDown stores each of its slots' rows into every rank's arena (peer[j] + out_offset,
    // [max_k + shared][dyn_rows] floats) instead of combining; k_expert_combine sums them
    int rank, ranks;
    char *peer[kMaxPeers];
    size_t out_offset;
    int *err;
    unsigned long long *probe;     // tracing only (heavy.cu probe), else NULL
    unsigned long long wait_ns;    // how long a bounded wait may last
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(unsigned long long *b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool bar_try(unsigned long long *b, int parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(10000u)
        : "memory");
    return ok != 0;
}
// Bounded wait on one phase; false (and *err set) after `limit` ns.
__device__ __forceinline__ bool bar_wait(unsigned long long *b, int parity, int *err, uint64_t limit) {
    if (bar_try(b, parity)) return true;
    const uint64_t start = global_time_ns();
    for (;;) {
        if (bar_try(b, parity)) return true;
        if (global_time_ns() - start > limit) {
            atomicCAS(err, 0, 2);
            return false;
        }
    }
}
__device__ __forceinline__ void bar_arrive(unsigned long long *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void bar_expect(unsigned long long *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
// dst, src 16-byte aligned, bytes a multiple of 16 (checked on the host).
__device__ __forceinline__ void bulk(void *dst, const void *src, uint32_t bytes, unsigned long long *b,
                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(b)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }
__device__ __forceinline__ uint4 lds16(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_u32(p)));
    return v;
}

__host__ __device__ __forceinline__ int esize(int dtype) { return dtype == MR_DTYPE_F32 ? 4 : 2; }
__host__ __device__ __forceinline__ int piece_rows(const Args &a) {
    const int rb = a.cols * esize(a.dtype) * (a.mode == kSwiglu ? 2 : 1);
    const int p = kSlotBytes / rb;
    return p < 1 ? 1 : p < kMaxPieceRows ? p : kMaxPieceRows;
}
// A ring slot holds one piece: its bytes rounded up to 128 (down projections of
// 1408-wide BF16 rows: 4 x 2816 = 11264 bytes, so the ring holds more of them).
inline int slot_bytes(const Args &a) {
    const int bytes = piece_rows(a) * a.cols * esize(a.dtype) * (a.mode == kSwiglu ? 2 : 1);
    return (bytes + 127) & ~127;
}
__device__ __forceinline__ int slice_lo(int rows, int c, int g) {
    return static_cast<int>(static_cast<long long>(rows) * c / g);
}

// The CTA's pieces, in one fixed order (static segments, then routed slots in
// rank order), each a run of up to piece_rows(a) rows of one segment.
struct Piece {
    const char *w, *w2;  // first row of the piece (w2: kSwiglu up rows)
    int seg_index;       // static segment, or -1 for a routed slot
    int slot, row0, nrows;
    float *y;
};
template <typename F>
__device__ __forceinline__ void for_each_piece(const Args &a, bool dynamic, int active, F &&f) {
    const int P = piece_rows(a);
    const size_t rb = static_cast<size_t>(a.cols) * esize(a.dtype);
    const int c = blockIdx.x, g = gridDim.x;
    int n = 0;
    if (!dynamic) {
        for (int s = 0; s < a.nseg; ++s) {
            const Seg &sg = a.seg[s];
            const int lo = slice_lo(sg.rows, c, g), hi = slice_lo(sg.rows, c + 1, g);
            for (int r = lo; r < hi; r += P) {
                Piece p{static_cast<const char *>(sg.w) + r * rb,
                        sg.w2 ? static_cast<const char *>(sg.w2) + r * rb : nullptr, s, sg.slot, r, min(P, hi - r),
                        sg.y};
                f(n++, p);
            }
        }
        return;
    }
    for (int s = 0; s < a.nseg; ++s) {
        const int lo = slice_lo(a.seg[s].rows, c, g), hi = slice_lo(a.seg[s].rows, c + 1, g);
        n += (hi - lo + P - 1) / P;
    }
    const int lo = slice_lo(a.dyn_rows, c, g), hi = slice_lo(a.dyn_rows, c + 1, g);
    for (int k = 0; k < active; ++k) {
        const int e = a.chosen[k];
        if (e < 0 || e >= a.experts) {  // never index outside the expert table
            atomicCAS(a.err, 0, 4);
            return;
        }
        if (a.ranks > 1 && e % a.ranks != a.rank) continue;  // another rank's expert
        const char *w = static_cast<const char *>(a.dyn_w[e]);
        const char *w2 = a.dyn_w2 ? static_cast<const char *>(a.dyn_w2[e]) : nullptr;
        for (int r = lo; r < hi; r += P) {
            Piece p{w + r * rb, w2 ? w2 + r * rb : nullptr, -1, k, r, min(P, hi - r), nullptr};
            f(n++, p);
        }
    }
}

// One 16-byte chunk of weights widened to float: kChunkCols columns, in
// column order (BF16 / F16: the low half of each 32-bit word first).
template <int DT>
constexpr int kChunkCols = DT == MR_DTYPE_F32 ? 4 : 8;
template <int DT>
__device__ __forceinline__ void widen(const uint4 &w, float (&v)[kChunkCols<DT>]) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (DT == MR_DTYPE_F32) {
            v[i] = __uint_as_float(u[i]);
        } else if (DT == MR_DTYPE_BF16) {
            v[2 * i] = __uint_as_float(u[i] << 16);
            v[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
        } else {
            v[2 * i] = __half2float(__ushort_as_half(static_cast<uint16_t>(u[i] & 0xffffu)));
            v[2 * i + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(u[i] >> 16)));
        }
    }
}
// The inputs of chunk c: columns 8c..8c+3 at xlo + 4c, 8c+4..8c+7 at xhi + 4c
// (F32: 4c..4c+3 at xlo + 4c).
template <int DT>
__device__ __forceinline__ void chunk_x(const float *xlo, const float *xhi, int c, float (&v)[kChunkCols<DT>]) {
    const float4 a = *reinterpret_cast<const float4 *>(xlo + 4 * c);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = a.z;
    v[3] = a.w;
    if (DT != MR_DTYPE_F32) {
        const float4 b = *reinterpret_cast<const float4 *>(xhi + 4 * c);
        v[4] = b.x;
        v[5] = b.y;
        v[6] = b.z;
        v[7] = b.w;
    }
}
// A row's running sums (one per column of a chunk) summed pairwise, then over the warp.
template <int DT>
__device__ __forceinline__ float fold(const float (&a)[kChunkCols<DT>]) {
    float s = (a[0] + a[1]) + (a[2] + a[3]);
    if (DT != MR_DTYPE_F32) s = s + ((a[4] + a[5]) + (a[6] + a[7]));
    return warp_sum(s);
}

// Dot products of n (<= kMaxPieceRows) consecutive rows of one slot with x.
// Lane l takes the 16-byte chunks l, l + 32, ...; each row keeps one running
// sum per column of a chunk, so a chunk's FMAs are independent of one another
// (a single chain per row left the warps waiting on FMA latency with two warps
// per scheduler); the sums fold pairwise at the end.  Every lane gets the sums.
template <int DT>
__device__ __forceinline__ void rows_dot(const char *slot, int n, int row_bytes, int nv, const float *xlo,
                                         const float *xhi, float (&y)[kMaxPieceRows]) {
    constexpr int W = kChunkCols<DT>;
    const int lane = threadIdx.x & 31;
    float acc[kMaxPieceRows][W];
#pragma unroll
    for (int r = 0; r < kMaxPieceRows; ++r)
#pragma unroll
        for (int k = 0; k < W; ++k) acc[r][k] = 0.f;
    for (int c = lane; c < nv; c += 32) {
        float x[W];
        chunk_x<DT>(xlo, xhi, c, x);
#pragma unroll
        for (int r = 0; r < kMaxPieceRows; ++r) {
            if (r >= n) break;
            float w[W];
            widen<DT>(lds16(slot + r * row_bytes + 16 * c), w);
#pragma unroll
            for (int k = 0; k < W; ++k) acc[r][k] = fmaf(w[k], x[k], acc[r][k]);
        }
    }
#pragma unroll
    for (int r = 0; r < kMaxPieceRows; ++r) y[r] = fold<DT>(acc[r]);
}

// x (n floats) into the layout the dot products read: two planes for 16-bit
// weights (columns 8c..8c+3 of chunk c at lo + 4c, 8c+4..8c+7 at hi + 4c,
// hi = lo + n/2), plain for F32.  With `norm`, RMSNorm(x, gain) computed by
// the 256 consumer threads exactly as stage_input does.
__device__ __forceinline__ int plane_index(int j, int n, bool split) {
    return split ? (j >> 3) * 4 + (j & 3) + ((j & 4) ? n / 2 : 0) : j;
}
constexpr int kGainRegs = 16;  // gains held per thread from before the dependency wait (n <= 4096)

// The norm gains this thread applies (elements t, t + 256, ...), loaded before
// the dependency wait: they are weights, which no kernel writes.
__device__ __forceinline__ void load_gains(const void *gain, int gain_dtype, int n, float (&g)[kGainRegs]) {
#pragma unroll
    for (int k = 0; k < kGainRegs; ++k) {
        const int i = threadIdx.x + k * kConsumers;
        g[k] = (gain && i < n) ? load_weight(gain, gain_dtype, i) : 1.0f;
    }
}

__device__ void stage(const float *x, int n, bool norm, const void *gain, int gain_dtype, const float (&g)[kGainRegs],
                      float eps, bool split, float *xs, float *red) {
    const int t = threadIdx.x;
    float ss = 0.f;
    const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (vec) {
#pragma unroll 4
        for (int i = 4 * t; i < n; i += 4 * kConsumers) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + i));
            xs[plane_index(i, n, split)] = v.x;
            xs[plane_index(i + 1, n, split)] = v.y;
            xs[plane_index(i + 2, n, split)] = v.z;
            xs[plane_index(i + 3, n, split)] = v.w;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
    } else {
#pragma unroll 4
        for (int i = t; i < n; i += kConsumers) {
            const float v = __ldcg(x + i);
            xs[plane_index(i, n, split)] = v;
            ss = fmaf(v, v, ss);
        }
    }
    if (!norm) return;  // the caller synchronises the consumers
    ss = warp_sum(ss);
    if ((t & 31) == 0) red[t >> 5] = ss;
    consumers_sync();
    float total = 0.f;
    for (int w = 0; w < kConsumerWarps; ++w) total += red[w];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(FADD(__fdiv_rn(total, static_cast<float>(n)), eps)));
#pragma unroll
    for (int k = 0; k < kGainRegs; ++k) {
        const int i = t + k * kConsumers;
        if (i < n) {
            const int at = plane_index(i, n, split);
            xs[at] = FMUL(FMUL(xs[at], scale), g[k]);
        }
    }
    for (int i = t + kGainRegs * kConsumers; i < n; i += kConsumers) {
        const float gv = gain ? load_weight(gain, gain_dtype, i) : 1.0f;
        const int at = plane_index(i, n, split);
        xs[at] = FMUL(FMUL(xs[at], scale), gv);
    }
}

// The down projection's inputs: the act rows of the active slots (routed
// 0 .. active-1, shared max_k ..), all loads of all rows in one pass.
__device__ void stage_acts(const Args &a, int active, bool split, float *xs) {
    const int slots_total = a.max_k + a.shared, n = a.cols, q = n / 4, total = slots_total * q;
    constexpr int kBatch = 8;  // loads in flight per thread before the first store
    for (int i0 = threadIdx.x; i0 < total; i0 += kBatch * kConsumers) {
        float4 v[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int i = i0 + b * kConsumers, k = i / q;
            const bool live = i < total && !(k >= active && k < a.max_k);
            v[b] = live ? __ldcg(reinterpret_cast<const float4 *>(a.acts + static_cast<size_t>(k) * n + 4 * (i % q)))
                        : float4{};
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int i = i0 + b * kConsumers, k = i / q, c = 4 * (i % q);
            if (i >= total || (k >= active && k < a.max_k)) continue;
            float *dst = xs + static_cast<size_t>(k) * n;
            dst[plane_index(c, n, split)] = v[b].x;
            dst[plane_index(c + 1, n, split)] = v[b].y;
            dst[plane_index(c + 2, n, split)] = v[b].z;
            dst[plane_index(c + 3, n, split)] = v[b].w;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(kThreads, 1) k_stream(Args a) {
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_trigger();
    const int S = a.slots;
    unsigned long long *full = reinterpret_cast<unsigned long long *>(smem);
    unsigned long long *empty = full + kMaxSlots;
    volatile int *issued_count = reinterpret_cast<volatile int *>(empty + kMaxSlots);  // pieces issued so far
    float *red = reinterpret_cast<float *>(empty + kMaxSlots) + 4;                     // 32 floats
    float *outs = red + 32;                                                // kDown: [slots_total][rows per CTA]
    const int slots_total = a.max_k + a.shared;
    const int rows_cta = a.mode == kDown    ? (a.dyn_rows + gridDim.x - 1) / gridDim.x + 1
                         : a.residual ? (a.seg[0].rows + gridDim.x - 1) / gridDim.x + 1
                                      : 0;
    float *xs = outs + ((max(slots_total, 1) * rows_cta + 31) & ~31);
    const int ninputs = a.mode == kDown ? slots_total : 1;
    unsigned char *ring = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(xs + static_cast<size_t>(ninputs) * a.cols) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_bytes = a.cols * esize(a.dtype);
    const int pair = a.mode == kSwiglu ? 2 : 1;
    if (threadIdx.x == 0) probe(a.probe, kProbeStart);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], 1);
        }
        *issued_count = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumerWarps) {  // ---- producer ----
        if (lane != 0) return;
        const uint64_t policy = evict_first();
        bool ok = true;
        int issued = 0;
        auto issue = [&](int n, const Piece &p) {
            if (!ok) return;
            const int s = n % S;
            if (n >= S && !bar_wait(&empty[s], ((n / S) - 1) & 1, a.err, a.wait_ns)) {
                ok = false;
                return;
            }
            const uint32_t bytes = static_cast<uint32_t>(p.nrows * row_bytes);
            unsigned char *dst = ring + static_cast<size_t>(s) * a.slot_bytes;
            bar_expect(&full[s], bytes * pair);
            bulk(dst, p.w, bytes, &full[s], policy);
            if (pair == 2) bulk(dst + bytes, p.w2, bytes, &full[s], policy);
            issued = n + 1;
            *issued_count = issued;
        };
        for_each_piece(a, false, 0, issue);
        pdl_wait();
        if (a.mode != kPlain) for_each_piece(a, true, min(max(*a.active, 0), a.max_k), issue);
        // every copy issued must land before the CTA exits (the consumers have
        // normally waited for them all; after an error, wait here, bounded)
        for (int n = max(0, issued - S); n < issued; ++n)
            if (!bar_wait(&full[n % S], (n / S) & 1, a.err, a.wait_ns)) break;
        return;
    }

    // ---- consumers ----
    float gains[kGainRegs];
    if (a.mode != kDown && a.norm) load_gains(a.gain, a.gain_dtype, a.cols, gains);
    pdl_wait();
    if (threadIdx.x == 0) probe(a.probe, kProbeWaited);
    const int active = a.mode == kPlain ? 0 : min(max(*a.active, 0), a.max_k);
    const bool split = DT != MR_DTYPE_F32;
    if (a.mode == kDown) {
        stage_acts(a, active, split, xs);
    } else {
        stage(a.x, a.cols, a.norm != 0, a.gain, a.gain_dtype, gains, a.eps, split, xs, red);
        if (a.residual)  // the residual rows this CTA updates (one segment), read while staging
            for (int i = threadIdx.x; i < slice_lo(a.seg[0].rows, blockIdx.x + 1, gridDim.x) -
                                             slice_lo(a.seg[0].rows, blockIdx.x, gridDim.x);
                 i += kConsumers)
                outs[i] = __ldcg(a.seg[0].y + slice_lo(a.seg[0].rows, blockIdx.x, gridDim.x) + i);
    }
    consumers_sync();
    if (threadIdx.x == 0) probe(a.probe, kProbeStaged);
    const int nv = row_bytes / 16;
    const int lo_dyn = slice_lo(a.dyn_rows, blockIdx.x, gridDim.x);
    bool ok = true;
    auto consume = [&](int n, const Piece &p) {
        if (!ok || n % kConsumerWarps != warp) return;
        const int s = n % S;
        if (*issued_count <= n) {  // piece n's phase is armed only once it is issued
            const uint64_t start = global_time_ns();
            while (*issued_count <= n)
                if (global_time_ns() - start > a.wait_ns) {
                    atomicCAS(a.err, 0, 2);
                    ok = false;
                    return;
                }
        }
        if (!bar_wait(&full[s], (n / S) & 1, a.err, a.wait_ns)) {
            ok = false;
            return;
        }
        const unsigned char *slot = ring + static_cast<size_t>(s) * a.slot_bytes;
        const float *x = a.mode == kDown ? xs + static_cast<size_t>(p.slot) * a.cols : xs;
        const float *xhi = x + a.cols / 2;
        float y[kMaxPieceRows];
        if (a.mode == kSwiglu) {  // rows: gate r .. r+n-1, then up r .. r+n-1 (n = 1 for 4096-wide rows)
            for (int r = 0; r < p.nrows; ++r) {
                const char *gp = reinterpret_cast<const char *>(slot) + r * row_bytes;
                const char *base = gp;
                float gu[kMaxPieceRows];
                // gate row r and up row r share the x reads (rows_dot's running sums)
                const int off = p.nrows * row_bytes;
                {
                    constexpr int W = kChunkCols<DT>;
                    float ag[W], au[W];
#pragma unroll
                    for (int k = 0; k < W; ++k) ag[k] = au[k] = 0.f;
                    for (int c = lane; c < nv; c += 32) {
                        float xv[W], wg[W], wu[W];
                        chunk_x<DT>(x, xhi, c, xv);
                        widen<DT>(lds16(base + 16 * c), wg);
                        widen<DT>(lds16(base + off + 16 * c), wu);
#pragma unroll
                        for (int k = 0; k < W; ++k) {
                            ag[k] = fmaf(wg[k], xv[k], ag[k]);
                            au[k] = fmaf(wu[k], xv[k], au[k]);
                        }
                    }
                    gu[0] = fold<DT>(ag);
                    gu[1] = fold<DT>(au);
                }
                if (lane == 0)
                    a.act_out[static_cast<size_t>(p.slot) * a.dyn_rows + p.row0 + r] =
                        FMUL(__fdiv_rn(gu[0], FADD(1.0f, expf(-gu[0]))), gu[1]);
            }
        } else {
            rows_dot<DT>(reinterpret_cast<const char *>(slot), p.nrows, row_bytes, nv, x, xhi, y);
            if (lane == 0) {
                for (int r = 0; r < p.nrows; ++r) {
                    if (a.mode == kDown) {
                        outs[p.slot * rows_cta + (p.row0 - lo_dyn) + r] = y[r];
                    } else if (a.residual) {
                        const int at = p.row0 + r - slice_lo(a.seg[0].rows, blockIdx.x, gridDim.x);
                        p.y[p.row0 + r] = FADD(outs[at], FMUL(a.scale, y[r]));
                    } else {
                        p.y[p.row0 + r] = y[r];
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) bar_arrive(&empty[s]);
    };
    for_each_piece(a, false, 0, consume);
    if (a.mode != kPlain) for_each_piece(a, true, active, consume);
    if (a.probe && lane == 0) probe(a.probe, kProbeMain);
    if (a.mode != kDown) {
        if (a.probe && lane == 0) probe(a.probe, kProbeExit);
        return;
    }
    // rank-order combine of this CTA's output rows (k_expert_combine's arithmetic)
    consumers_sync();
    if (!ok) return;
    const int hi_dyn = slice_lo(a.dyn_rows, blockIdx.x + 1, gridDim.x);
    if (a.ranks > 1) {  // expert parallel: this rank's slots' rows to every rank
        for (int i = threadIdx.x; i < hi_dyn - lo_dyn; i += kConsumers) {
            auto put = [&](int slot) {
                const float v = outs[slot * rows_cta + i];
                const size_t at = a.out_offset + (static_cast<size_t>(slot) * a.dyn_rows + lo_dyn + i) * sizeof(float);
                for (int j = 0; j < a.ranks; ++j) *reinterpret_cast<float *>(a.peer[j] + at) = v;
            };
            for (int s = 0; s < a.nseg; ++s) put(a.seg[s].slot);
            for (int k = 0; k < active; ++k)
                if (a.chosen[k] % a.ranks == a.rank) put(k);
        }
        __threadfence_system();  // before k_moe_publish raises this rank's flag
        return;
    }
    for (int i = threadIdx.x; i < hi_dyn - lo_dyn; i += kConsumers) {
        float res = 0.f;
        for (int k = 0; k < active; ++k) res = FADD(res, FMUL(a.weights[k], outs[k * rows_cta + i]));
        for (int j = 0; j < a.shared; ++j) res = FADD(res, FMUL(a.shared_scale, outs[(a.max_k + j) * rows_cta + i]));
        float *xr = a.xres + lo_dyn + i;
        *xr = FADD(*xr, FMUL(a.scale, res));
    }
    if (threadIdx.x == 0) probe(a.probe, kProbeExit);
}

// Shared memory a launch needs besides the ring; the ring gets the rest of `budget`.
inline size_t fixed_smem(const Args &a, int grid) {
    const int slots_total = a.max_k + a.shared;
    const int rows_cta = a.mode == kDown ? (a.dyn_rows + grid - 1) / grid + 1
                         : a.residual    ? (a.seg[0].rows + grid - 1) / grid + 1
                                         : 0;
    const int ninputs = a.mode == kDown ? slots_total : 1;
    return 2 * kMaxSlots * sizeof(unsigned long long) + (4 + 32) * sizeof(float) +
           static_cast<size_t>((std::max(slots_total, 1) * rows_cta + 31) & ~31) * sizeof(float) +
           static_cast<size_t>(ninputs) * a.cols * sizeof(float) + 128;
}

}  // namespace stream
