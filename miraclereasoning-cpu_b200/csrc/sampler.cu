// Seeded top-k / top-p sampling on the device, the reference's procedure
// (model.py:343-352) to the bit:
//
//   order  = argsort(-logits, stable)[:top_k]           (top_k 0: every token)
//   scores = float64(logits[order]) / temperature
//   probs  = exp(scores - max); probs /= sum(probs)     (NumPy's pairwise sum)
//   cutoff = min(len, searchsorted(cumsum(probs), top_p) + 1)
//   token  = Generator.choice(order[:cutoff], p = probs[:cutoff] / sum(probs[:cutoff]))
//
// and Generator.choice(p) is: cdf = cumsum(p); cdf /= cdf[-1]; u = random();
// index = searchsorted(cdf, u, side="right"), random() being one PCG64 draw
// (128-bit LCG step, XSL-RR output, 53 bits to a double).  The host hands over
// the state of `numpy.random.default_rng(seed)` (sampler_seed); nothing else
// crosses to the host per token.  Temperature 0 takes order[0], NumPy's argmax
// (the first of equal maxima).
//
// The sort is a stable radix sort of the logits' order-preserving integer keys
// (CUB; -0 counted as +0, as NumPy compares them equal); the float64 work is
// one warp: the exponentials in parallel, the sums and prefix sums serially in
// NumPy's order (they decide the token).  A non-finite logit stops the
// generation, as the reference raises on it (model.py:331-332).
#include <cub/device/device_radix_sort.cuh>

#include <cstdint>

#include "sampler.cuh"

namespace mr {

struct SamplerState {
    unsigned long long state_hi, state_lo, inc_hi, inc_lo;  // PCG64
    int count;      // tokens produced
    int stopped;    // EOS, max_new or a non-finite logit
    int nonfinite;
};

struct Sampler {
    int vocab = 0;
    unsigned *keys_in = nullptr, *keys_out = nullptr;
    int *idx_in = nullptr, *idx_out = nullptr;
    double *probs = nullptr;
    void *temp = nullptr;
    size_t temp_bytes = 0;
    SamplerState *st = nullptr;
};

namespace {

// 128-bit multiply-add of the LCG: state = state * M + inc (mod 2^128).
__device__ __forceinline__ void pcg_step(SamplerState &s) {
    const unsigned long long m_hi = 0x2360ED051FC65DA4ull, m_lo = 0x4385DF649FCCF645ull;
    const unsigned long long lo = s.state_lo * m_lo;
    const unsigned long long hi = __umul64hi(s.state_lo, m_lo) + s.state_lo * m_hi + s.state_hi * m_lo;
    const unsigned long long nlo = lo + s.inc_lo;
    s.state_hi = hi + s.inc_hi + (nlo < lo ? 1ull : 0ull);
    s.state_lo = nlo;
}
__device__ __forceinline__ double next_double(SamplerState &s) {
    pcg_step(s);
    const unsigned long long x = s.state_hi ^ s.state_lo;
    const unsigned r = static_cast<unsigned>(s.state_hi >> 58);
    const unsigned long long out = (x >> r) | (x << ((64u - r) & 63u));
    return static_cast<double>(out >> 11) * (1.0 / 9007199254740992.0);
}

// NumPy's pairwise summation of float64: identity start; up to 8 values in
// order; up to 128 in eight running sums combined as ((r0+r1)+(r2+r3)) +
// ((r4+r5)+(r6+r7)) plus the tail; above that the two halves (the first a
// multiple of 8) summed apart and added.  Evaluated without recursion: an
// explicit stack visits the halves in the same order (depth <= 32 covers 2^36).
__device__ double pairwise_leaf(const double *a, int n) {
    if (n < 8) {
        double res = 0.0;
        for (int i = 0; i < n; ++i) res = __dadd_rn(res, a[i]);
        return res;
    }
    double r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
        for (int j = 0; j < 8; ++j) r[j] = __dadd_rn(r[j], a[i + j]);
    double res = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                           __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
    for (; i < n; ++i) res = __dadd_rn(res, a[i]);
    return res;
}
__device__ double pairwise_sum(const double *a, int n) {
    constexpr int kDepth = 32;
    int start[kDepth], len[kDepth], phase[kDepth];
    double left[kDepth];
    int top = 0;
    start[0] = 0;
    len[0] = n;
    phase[0] = 0;
    double value = 0.0;  // the value of the frame just finished
    while (top >= 0) {
        const int m = len[top];
        if (m <= 128) {
            value = pairwise_leaf(a + start[top], m);
            --top;
        } else {
            const int n2 = m / 2 - (m / 2) % 8;
            if (phase[top] == 0) {  // the first half
                phase[top] = 1;
                start[top + 1] = start[top];
                len[top + 1] = n2;
                phase[top + 1] = 0;
                ++top;
                continue;
            }
            if (phase[top] == 1) {  // the second half, the first's value kept
                phase[top] = 2;
                left[top] = value;
                start[top + 1] = start[top] + n2;
                len[top + 1] = m - n2;
                phase[top + 1] = 0;
                ++top;
                continue;
            }
            value = __dadd_rn(left[top], value);
            --top;
        }
        // a finished frame hands its value to its parent (phase 1 or 2 there)
    }
    return value;
}

// Descending logits as ascending keys (ties keep their order: the sort is stable).
__global__ void k_keys(const float *logits, int V, unsigned *keys, int *idx, SamplerState *s) {
    if (s->stopped) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        float v = logits[i];
        if (!isfinite(v)) atomicExch(&s->nonfinite, 1);
        if (v == 0.0f) v = 0.0f;
        const unsigned b = __float_as_uint(v);
        const unsigned ordered = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
        keys[i] = ~ordered;
        idx[i] = i;
    }
}

// One warp: the token from the sorted order; its id into *token_slot and out[count].
__global__ void k_pick(const float *logits, const int *order, int V, int top_k, double temperature, double top_p,
                       double *probs, SamplerState *s, int *token_slot, int *out, int eos, int max_new,
                       int *stop_flag) {
    const int lane = threadIdx.x;
    if (s->stopped) return;
    if (s->nonfinite) {
        if (lane == 0) {
            s->stopped = 1;
            if (stop_flag) *stop_flag = 1;
        }
        return;
    }
    int token;
    if (temperature == 0.0) {
        token = order[0];
    } else {
        const int K = top_k > 0 && top_k < V ? top_k : V;
        const double top = __ddiv_rn(static_cast<double>(logits[order[0]]), temperature);
        for (int i = lane; i < K; i += 32)
            probs[i] = exp(__dsub_rn(__ddiv_rn(static_cast<double>(logits[order[i]]), temperature), top));
        __syncwarp();
        __shared__ double total;
        if (lane == 0) total = pairwise_sum(probs, K);
        __syncwarp();
        for (int i = lane; i < K; i += 32) probs[i] = __ddiv_rn(probs[i], total);
        __syncwarp();
        if (lane != 0) return;
        // cutoff: the first prefix sum >= top_p (searchsorted, side left), plus one
        int cutoff = K;
        double c = 0.0;
        for (int i = 0; i < K; ++i) {
            c = __dadd_rn(c, probs[i]);
            if (c >= top_p) {
                cutoff = i + 1;
                break;
            }
        }
        // choice: p = probs / sum; cdf = cumsum(p) / cdf[-1]; first cdf > u (side right)
        const double psum = pairwise_sum(probs, cutoff);
        double last = 0.0;
        for (int i = 0; i < cutoff; ++i) last = __dadd_rn(last, __ddiv_rn(probs[i], psum));
        const double u = next_double(*s);
        int pick = cutoff - 1;
        double run = 0.0;
        for (int i = 0; i < cutoff; ++i) {
            run = __dadd_rn(run, __ddiv_rn(probs[i], psum));
            if (__ddiv_rn(run, last) > u) {
                pick = i;
                break;
            }
        }
        token = order[pick];
    }
    if (lane != 0) return;
    out[s->count] = token;
    s->count += 1;
    *token_slot = token;
    if (token == eos || s->count >= max_new) {
        s->stopped = 1;
        if (stop_flag) *stop_flag = 1;
    }
}

}  // namespace

int sampler_create(int vocab, Sampler **out) {
    Sampler *s = new Sampler();
    s->vocab = vocab;
    auto fail = [&](cudaError_t e) {
        sampler_destroy(s);
        return set_error(MR_ERR_CUDA, "sampler allocation failed: %s", cudaGetErrorString(e));
    };
    cudaError_t e;
    if ((e = cudaMalloc(&s->keys_in, sizeof(unsigned) * vocab)) != cudaSuccess ||
        (e = cudaMalloc(&s->keys_out, sizeof(unsigned) * vocab)) != cudaSuccess ||
        (e = cudaMalloc(&s->idx_in, sizeof(int) * vocab)) != cudaSuccess ||
        (e = cudaMalloc(&s->idx_out, sizeof(int) * vocab)) != cudaSuccess ||
        (e = cudaMalloc(&s->probs, sizeof(double) * vocab)) != cudaSuccess ||
        (e = cudaMalloc(&s->st, sizeof(SamplerState))) != cudaSuccess)
        return fail(e);
    if ((e = cub::DeviceRadixSort::SortPairs(nullptr, s->temp_bytes, s->keys_in, s->keys_out, s->idx_in, s->idx_out,
                                             vocab)) != cudaSuccess ||
        (e = cudaMalloc(&s->temp, s->temp_bytes)) != cudaSuccess)
        return fail(e);
    *out = s;
    return MR_OK;
}

void sampler_destroy(Sampler *s) {
    if (!s) return;
    for (void *p : {static_cast<void *>(s->keys_in), static_cast<void *>(s->keys_out), static_cast<void *>(s->idx_in),
                    static_cast<void *>(s->idx_out), static_cast<void *>(s->probs), s->temp,
                    static_cast<void *>(s->st)})
        if (p) cudaFree(p);
    delete s;
}

int sampler_seed(Sampler *s, cudaStream_t stream, const unsigned long long pcg[4]) {
    SamplerState h{pcg[0], pcg[1], pcg[2], pcg[3], 0, 0, 0};
    MR_CUDA_TRY(cudaMemcpyAsync(s->st, &h, sizeof(h), cudaMemcpyHostToDevice, stream));
    return MR_OK;
}

int sampler_step(Sampler *s, cudaStream_t stream, const float *logits, const SampleParams &p, int *token_slot,
                 int *out, int *stop_flag) {
    k_keys<<<64, 256, 0, stream>>>(logits, s->vocab, s->keys_in, s->idx_in, s->st);
    MR_CUDA_TRY(cudaGetLastError());
    MR_CUDA_TRY(cub::DeviceRadixSort::SortPairs(s->temp, s->temp_bytes, s->keys_in, s->keys_out, s->idx_in, s->idx_out,
                                                s->vocab, 0, 32, stream));
    k_pick<<<1, 32, 0, stream>>>(logits, s->idx_out, s->vocab, p.top_k, p.temperature, p.top_p, s->probs, s->st,
                                 token_slot, out, p.eos, p.max_new, stop_flag);
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

int sampler_result(Sampler *s, cudaStream_t stream, int *count, int *nonfinite) {
    SamplerState h;
    MR_CUDA_TRY(cudaMemcpyAsync(&h, s->st, sizeof(h), cudaMemcpyDeviceToHost, stream));
    MR_CUDA_TRY(cudaStreamSynchronize(stream));
    *count = h.count;
    *nonfinite = h.nonfinite;
    return MR_OK;
}

}  // namespace mr
