// Whole-model engine, host side: tensor registry (the canonical names and
// shapes of weights.py expected_shapes, weights.py:211-245), HBM residency of
// the stored bytes, the per-step phase plan, and the launch loop behind
// mr_model_step / prefill / generate.
//
// Replaces the reference's per-op Python dispatch (model.py:257-312), its
// per-op clCreateBuffer/clEnqueueNDRangeKernel traffic (opencl.py:178-239)
// and its LRU weight cache (weights.py:258-297).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <fcntl.h>
#include <unistd.h>

#include "engine.cuh"
#include "heavy.cuh"
#include "prefill.cuh"
#include "aux_step.cuh"
#include "sampler.cuh"

namespace mr {

__global__ void decode_step_kernel(const Phase *__restrict__ phases, int nphases, StepState *st, StepControl ctl);
size_t decode_control_bytes();

namespace {

struct TensorSlot {
    std::vector<int64_t> shape;
    int dtype = -1;
    void *ptr = nullptr;
    size_t bytes = 0;
};

bool is_gqa_family(int f) {
    return f == MR_FAMILY_FLASHNANO_15 || f == MR_FAMILY_FLASHNANO_17 || f == MR_FAMILY_FLASHLITE_20;
}

// FlashLighting with no memory slots (the family default) compacts its latent
// cache by dropping the oldest row (model.py:171-176): attention then covers
// the newest `window` latents, whose keys and values (normed, rotated at the
// latent's own position) never change once computed.  The engine keeps them in
// a ring of `window` rows, computing one row per token, which gives the same
// keys and values the reference recomputes from the stored latents every step.
bool is_lighting_ring(const mr_model_config &c) {
    return c.family == MR_FAMILY_FLASHLIGHTING_20 && c.memory_slots == 0 && c.window > 0;
}

// FlashLighting with memory slots: the same ring for the window, and memory rows
// (absorbed and merged latents) that the work between steps keeps (aux_step.cuh).
bool is_lighting_memory(const mr_model_config &c) {
    return c.family == MR_FAMILY_FLASHLIGHTING_20 && c.memory_slots > 0 && c.window > 0;
}
bool is_lighting(const mr_model_config &c) { return is_lighting_ring(c) || is_lighting_memory(c); }

// flashnano-1.6: grouped-query attention plus chunk relays (aux_step.cuh).
bool is_cbr(const mr_model_config &c) {
    return c.family == MR_FAMILY_FLASHNANO_16 && c.cbr_chunk_size > 0 && c.cbr_slots > 0;
}

// Families the persistent decode kernel plans (the others step on the host).
bool is_engine_family(const mr_model_config &c) {
    return is_gqa_family(c.family) || is_lighting(c) || is_cbr(c);
}

size_t dtype_size(int dtype) { return dtype == MR_DTYPE_F32 ? 4 : 2; }

// ---- synthetic weights (counter hash, bit-identical to synthetic.py) -------------
__device__ __forceinline__ uint64_t splitmix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_fill_hash_bf16(uint16_t *out, size_t n, uint64_t key, float scale) {
    const uint64_t golden = 0x9E3779B97F4A7C15ull, lanes = 0x0000FFFF0000FFFFull;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        uint64_t acc = 0;
        for (uint64_t w = 0; w < 3; ++w) {
            const uint64_t z = splitmix(((3ull * i + w) * golden) ^ key);
            acc += z & lanes;
            acc += (z >> 16) & lanes;
        }
        const uint64_t total = (acc & 0xFFFFFFFFull) + (acc >> 32);
        const float centred = static_cast<float>(static_cast<int64_t>(total) - 6 * 65536);
        const uint32_t bits = __float_as_uint(__fmul_rn(centred, scale));
        out[i] = static_cast<uint16_t>((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
    }
}

__global__ void k_fill_value(void *out, int dtype, size_t n, float value) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        if (dtype == MR_DTYPE_F32) {
            static_cast<float *>(out)[i] = value;
        } else if (dtype == MR_DTYPE_BF16) {
            const uint32_t bits = __float_as_uint(value);
            static_cast<uint16_t *>(out)[i] = static_cast<uint16_t>((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
        } else {
            static_cast<__half *>(out)[i] = __float2half_rn(value);
        }
    }
}

uint64_t host_splitmix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

}  // namespace
}  // namespace mr

using namespace mr;

struct mr_model {
    mr_context *ctx = nullptr;
    mr_model_config cfg{};
    std::vector<int> layer_kvh, layer_window;
    std::vector<float> inv_freq;
    std::map<std::string, TensorSlot> tensors;
    std::vector<void *> allocations;
    bool finalized = false;
    bool failed = false;
    bool op_path = false;  // no decode plan: the token step runs on the host over the op kernels
    HeavyEngine *heavy = nullptr;  // heavy-medium-2.0: the token step as kernel launches (heavy.cu)
    unsigned long long wait_limit_ns = 0;  // device waits give up after this (0: the kernels' 2 s)
    // mr_model_load_file: two page-locked staging buffers and the copy out of each
    unsigned char *staging[2] = {nullptr, nullptr};
    cudaEvent_t staged[2] = {nullptr, nullptr};
    int withhold_phase = -1;               // fault injection for tests (mr_model_inject_fault)
    int position = 0;
    int grid = 0;
    // device buffers
    float *d_inv_freq = nullptr;
    Word *x = nullptr, *q_raw = nullptr, *k_raw = nullptr, *v_raw = nullptr, *ffn = nullptr;  // exchange words
    Word *latent = nullptr;  // FlashLighting: the layer's latent row
    Word *attn_out = nullptr;
    unsigned long long launches = 0;  // launches so far: each gets its own exchange tags
    float *logits = nullptr;
    int logits_rows = 0;
    Word *partial = nullptr;
    int scratch_floats = 0, attn_base = 0, ring_bytes = 0;
    int xres_skip = 0;              // CTAs owning no rows of the q/k/v, o and down phases
    size_t smem_bytes = 0;
    PieceDesc *d_pieces = nullptr;
    GroupTable *d_groups = nullptr;
    int *d_piece_count = nullptr;
    int piece_stride = 0;
    std::vector<float *> k_cache, v_cache;
    std::vector<int> cache_capacity;
    StepState *state = nullptr;
    int *feed = nullptr;
    int feed_capacity = 0;
    int *gen_out = nullptr;
    int gen_capacity = 0;
    Phase *d_phases = nullptr;
    std::vector<Phase> phases;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // page-locked host staging of a decode call: its token ids in, then the
    // device error word and the logits out, all queued before one synchronise
    int *h_ids = nullptr, *h_error = nullptr;
    float *h_logits = nullptr;
    static constexpr int kHostIds = 256;
    // tensor parallel: this rank of `ranks`; every exchange buffer lives in one arena
    // whose IPC handle the other ranks open (peer[j] = rank j's arena, mapped here)
    int rank = 0, ranks = 1;
    char *arena = nullptr;
    size_t arena_bytes = 0;
    char *peer[kMaxRanks] = {};
    bool peer_open[kMaxRanks] = {};
    bool connected = false;
    Word *best_slots = nullptr;
    int xres_lo = 0, xres_n = 0;
    // flashnano-1.6 chunk relays / FlashLighting memory slots: the work between two
    // steps (aux_step.cuh), its layer table on the device and a host copy of it
    bool aux_on = false;
    aux::Model aux_model{};
    aux::Layer *aux_layers = nullptr;
    std::vector<aux::Layer> aux_host;
    int aux_kvh = 0;  // the most KV heads of any layer (grid of the projections)
    Sampler *sampler = nullptr;  // device sampling (sampler.cu), created on first use
    // batched prefill (prefill.cu): available for BF16 models of the engine families
    bool prefill_ok = false, prefill_on = true;
    PrefillModel pm{};
    PrefillWork pw{};
};

namespace {

void *device_alloc(mr_model *m, size_t bytes, int *rc) {
    void *p = nullptr;
    bytes = (bytes + 255) & ~size_t(255);
    cudaError_t err = cudaMalloc(&p, bytes ? bytes : 256);
    if (err != cudaSuccess) {
        *rc = cuda_error(err, "cudaMalloc");
        return nullptr;
    }
    m->allocations.push_back(p);
    return p;
}

// Canonical tensor names and shapes (weights.py expected_shapes).
void expected_tensors(mr_model *m) {
    const mr_model_config &c = m->cfg;
    const int64_t h = c.hidden_size, d = c.head_dim, q = (int64_t)c.query_heads * c.head_dim, f = c.ffn_dim;
    auto add = [&](const std::string &name, std::vector<int64_t> shape) { m->tensors[name].shape = shape; };
    add("embed", {c.vocab_size, h});
    add("norm", {h});
    if (!c.tie_embeddings) add("output", {c.vocab_size, h});
    const bool heavy = c.family == MR_FAMILY_HEAVY_MEDIUM_20, lighting = c.family == MR_FAMILY_FLASHLIGHTING_20;
    for (int i = 0; i < c.layers; ++i) {
        const std::string p = "layers." + std::to_string(i) + ".";
        const int64_t kv = (int64_t)m->layer_kvh[i] * d;
        add(p + "a_norm", {h});
        add(p + "q", {q, h});
        add(p + "o", {h, q});
        if (!lighting) add(p + "f_norm", {h});
        if (c.latent_dim) add(p + "latent", {c.latent_dim, h});
        if (heavy) {
            add(p + "kv_up", {2 * kv, c.latent_dim});
            add(p + "router.coarse.weight", {c.router_groups, h});
            add(p + "router.coarse.bias", {c.router_groups});
            add(p + "router.fine.weight", {c.routed_experts, h});
            add(p + "router.fine.bias", {c.routed_experts});
            add(p + "router.group_bias", {c.router_groups});
            add(p + "router.expert_bias", {c.routed_experts});
        } else {
            const int64_t inner = c.latent_dim ? c.latent_dim : h;
            add(p + "k", {kv, inner});
            add(p + "v", {kv, inner});
            if (c.qk_norm) {
                add(p + "q_norm", {d});
                add(p + "k_norm", {d});
            }
        }
        if (lighting) {
            add(p + "latent_norm", {c.latent_dim});
            add(p + "attention_gate", {1});
            add(p + "ffn_gate", {1});
        }
        if (c.family == MR_FAMILY_FLASHNANO_16) add(p + "cbr", {c.cbr_slots, h});
        std::vector<std::string> roots;
        if (heavy) {
            for (int e = 0; e < c.routed_experts; ++e) roots.push_back(p + "experts." + std::to_string(e) + ".");
            for (int e = 0; e < c.shared_experts; ++e) roots.push_back(p + "shared." + std::to_string(e) + ".");
        } else {
            roots.push_back(p + "ffn.");
        }
        for (auto &r : roots) {
            add(r + "gate", {f, h});
            add(r + "up", {f, h});
            add(r + "down", {h, f});
        }
    }
}

int check_tensor(mr_model *m, const char *name, int dtype, int ndim, const int64_t *shape, TensorSlot **out) {
    MR_REQUIRE(m && name, "NULL argument");
    MR_REQUIRE(!m->finalized, "model is finalized; tensors are immutable");
    auto it = m->tensors.find(name);
    MR_REQUIRE(it != m->tensors.end(), "unexpected tensor %s", name);
    MR_REQUIRE(dtype == MR_DTYPE_F32 || dtype == MR_DTYPE_F16 || dtype == MR_DTYPE_BF16, "%s: unsupported dtype %d",
               name, dtype);
    TensorSlot &t = it->second;
    bool same = ndim == (int)t.shape.size() && shape;
    for (int i = 0; same && i < ndim; ++i) same = shape[i] == t.shape[i];
    if (!same) {
        std::string want;
        for (auto v : t.shape) want += std::to_string(v) + ",";
        return set_error(MR_ERR_ARGUMENT, "%s: expected shape (%s)", name, want.c_str());
    }
    size_t n = 1;
    for (auto v : t.shape) n *= (size_t)v;
    const size_t bytes = n * dtype_size(dtype);
    if (!t.ptr || t.bytes != bytes) {
        int rc = MR_OK;
        t.ptr = device_alloc(m, bytes, &rc);
        if (rc) return rc;
    }
    t.bytes = bytes;
    t.dtype = dtype;
    *out = &t;
    return MR_OK;
}

const TensorSlot *tensor(mr_model *m, const std::string &name) {
    auto it = m->tensors.find(name);
    return it == m->tensors.end() ? nullptr : &it->second;
}

Segment segment(const TensorSlot *t, Word *out = nullptr) {
    Segment s{};
    s.w = t->ptr;
    s.dtype = t->dtype;
    s.rows = (int)t->shape[0];
    s.cols = (int)t->shape[1];
    s.out = out;
    return s;
}

Phase gemv_phase(int layer, const Word *in, const TensorSlot *norm_gain, float eps) {
    Phase ph{};
    ph.kind = PH_GEMV;
    ph.layer = layer;
    ph.gemv.input_kind = IN_VECTOR;
    ph.gemv.in = in;
    ph.gemv.in_back = 1;
    if (norm_gain) {
        ph.gemv.norm = 1;
        ph.gemv.norm_gain = norm_gain->ptr;
        ph.gemv.norm_gain_dtype = norm_gain->dtype;
        ph.gemv.norm_eps = eps;
    }
    return ph;
}

// Piece and group caps of a phase (bytes).  While a CTA's rows of the phase
// fit in half the ring (one group), pieces are at most a quarter of the ring
// and groups at most half.  Phases that stream more per CTA take groups of up
// to two thirds of the ring with pieces of at most a sixth: fewer group turns
// (each costs a barrier and a row table; -4% step time on FlashLite), and a
// group, the gain piece and a piece lost to a wrap still fit the ring together.
void phase_caps(const mr_model *m, const GemvPhase &g, int &piece_cap, int &group_cap) {
    const int ring = m->ring_bytes, n = m->grid - g.skip;
    long long per_cta = 0;
    int widest = 0;
    for (int i = 0; i < g.nseg; ++i) {
        const int row_bytes = g.seg[i].cols * (int)dtype_size(g.seg[i].dtype);
        per_cta += (long long)((g.seg[i].row_n + n - 1) / n) * row_bytes;
        widest = std::max(widest, row_bytes);
    }
    if (per_cta <= ring / 2 || widest > ring / 6) {
        piece_cap = ring / 4;
        group_cap = ring / 2;
    } else {
        piece_cap = ring / 6;
        group_cap = (int)((long long)ring * 2 / 3);
    }
}

// The attention phase of layer l: q words from `q_back` phases back, this
// token's k / v words from the phase just before.
int attn_phase(mr_model *m, int l, bool qk_norm, int q_back, Phase &at) {
    const mr_model_config &c = m->cfg;
    const std::string p = "layers." + std::to_string(l) + ".";
    at = Phase{};
    at.kind = PH_ATTN_GQA;
    at.layer = l;
    AttnPhase &a = at.attn;
    a.q_raw = m->q_raw;
    a.k_raw = m->k_raw;
    a.v_raw = m->v_raw;
    a.q_back = q_back;
    a.qk_norm = qk_norm;
    if (qk_norm) {
        const TensorSlot *qn = tensor(m, p + "q_norm"), *kn = tensor(m, p + "k_norm");
        if (qn->dtype != kn->dtype) return set_error(MR_ERR_ARGUMENT, "q_norm/k_norm dtypes differ");
        a.q_gain = qn->ptr;
        a.k_gain = kn->ptr;
        a.gain_dtype = qn->dtype;
    }
    a.norm_eps = c.norm_eps;
    a.heads = c.query_heads;
    a.kv_heads = m->layer_kvh[l];
    a.dim = c.head_dim;
    a.split_half = c.split_half_rope;
    a.inv_freq = m->d_inv_freq;
    a.k_cache = m->k_cache[l];
    a.v_cache = m->v_cache[l];
    a.capacity = m->cache_capacity[l];
    a.partial = m->partial;
    a.out = m->attn_out;
    return MR_OK;
}

// A one-element tensor (a FlashLighting gate) widened to float on the host.
int read_scalar(mr_model *m, const std::string &name, float &value) {
    const TensorSlot *t = tensor(m, name);
    MR_REQUIRE(t && t->ptr, "missing tensor %s", name.c_str());
    uint32_t raw = 0;
    MR_CUDA_TRY(cudaMemcpy(&raw, t->ptr, dtype_size(t->dtype), cudaMemcpyDeviceToHost));
    if (t->dtype == MR_DTYPE_F32) {
        memcpy(&value, &raw, 4);
    } else if (t->dtype == MR_DTYPE_BF16) {
        const uint32_t bits = raw << 16;
        memcpy(&value, &bits, 4);
    } else {
        __half h;
        memcpy(&h, &raw, 2);
        value = __half2float(h);
    }
    return MR_OK;
}

// FlashLighting layer (model.py:146-190, 272-278) on the ring form above.
// Both branches read the same RMSNorm(x): phases
//   1. q | latent       = W (a_norm x)
//   2. SwiGLU(gate, up) of a_norm x                        (independent of 1)
//   3. k | v            = W (latent_norm latent)
//   4. attention: q from phase 1, k / v from phase 3 (q_norm / k_norm + RoPE)
//   5. x += (residual_scale * attention_gate) * (W_o attended)   (kept in shared memory)
//   6. x += (residual_scale * ffn_gate) * (W_down ffn)            (published)
// The gates are weights read once here.  The reference forms
// x + s * (ag * o + fg * f); this sums the two scaled branches into x one at a
// time (a float32 rounding difference).  Only phase 6 publishes x, so no
// phase of the layer overwrites x words that phases 1 and 2 of another CTA may
// still be reading (phase 6 needs every CTA's phase-2 output first).
int plan_lighting_layer(mr_model *m, int l) {
    const mr_model_config &c = m->cfg;
    const std::string p = "layers." + std::to_string(l) + ".";
    const TensorSlot *embed = tensor(m, "embed");
    auto input = [&](Phase &ph, int back) {
        ph.gemv.in_back = back;
        if (l == 0) {
            ph.gemv.input_kind = IN_EMBED_ROW;
            ph.gemv.embed = embed->ptr;
            ph.gemv.embed_dtype = embed->dtype;
        }
    };
    Phase ql = gemv_phase(l, m->x, tensor(m, p + "a_norm"), c.norm_eps);
    input(ql, 1);
    ql.gemv.nseg = 2;
    ql.gemv.seg[0] = segment(tensor(m, p + "q"), m->q_raw);
    ql.gemv.seg[1] = segment(tensor(m, p + "latent"), m->latent);
    ql.gemv.epilogue = EPI_STORE;
    ql.gemv.skip = m->xres_skip;
    m->phases.push_back(ql);
    Phase gu = gemv_phase(l, m->x, tensor(m, p + "a_norm"), c.norm_eps);
    input(gu, 2);
    gu.gemv.nseg = 2;
    gu.gemv.seg[0] = segment(tensor(m, p + "ffn.gate"));
    gu.gemv.seg[1] = segment(tensor(m, p + "ffn.up"));
    gu.gemv.epilogue = EPI_SWIGLU;
    gu.gemv.out = m->ffn;
    m->phases.push_back(gu);
    Phase kv = gemv_phase(l, m->latent, tensor(m, p + "latent_norm"), c.norm_eps);
    kv.gemv.in_back = 2;
    kv.gemv.nseg = 2;
    kv.gemv.seg[0] = segment(tensor(m, p + "k"), m->k_raw);
    kv.gemv.seg[1] = segment(tensor(m, p + "v"), m->v_raw);
    kv.gemv.epilogue = EPI_STORE;
    kv.gemv.skip = m->xres_skip;
    if (is_lighting_memory(c)) {  // the raw latents, for rows that leave the window into memory
        kv.gemv.save_in = m->aux_host[l].lat_ring;
        kv.gemv.save_rows = m->cache_capacity[l];
    }
    m->phases.push_back(kv);
    Phase at;
    if (int rc = attn_phase(m, l, true, 3, at)) return rc;
    if (is_lighting_memory(c)) {  // the window ring, then the memory rows (model.py:160-165)
        at.attn.relay_k = m->aux_host[l].relay_k;
        at.attn.relay_v = m->aux_host[l].relay_v;
        at.attn.relay_count = m->aux_host[l].relay_count;
        at.attn.relay_capacity = m->aux_host[l].relay_cap;
    }
    m->phases.push_back(at);
    float ag = 0.f, fg = 0.f;
    if (int rc = read_scalar(m, p + "attention_gate", ag)) return rc;
    if (int rc = read_scalar(m, p + "ffn_gate", fg)) return rc;
    Phase o = gemv_phase(l, m->attn_out, nullptr, 0.f);
    o.gemv.nseg = 1;
    o.gemv.seg[0] = segment(tensor(m, p + "o"));
    o.gemv.epilogue = EPI_RESIDUAL_KEEP;
    o.gemv.scale = c.residual_scale * ag;
    o.gemv.x = m->x;
    o.gemv.skip = m->xres_skip;
    m->phases.push_back(o);
    Phase dn = gemv_phase(l, m->ffn, nullptr, 0.f);
    dn.gemv.in_back = 4;
    dn.gemv.nseg = 1;
    dn.gemv.seg[0] = segment(tensor(m, p + "ffn.down"));
    dn.gemv.epilogue = EPI_RESIDUAL;
    dn.gemv.scale = c.residual_scale * fg;
    dn.gemv.x = m->x;
    dn.gemv.skip = m->xres_skip;
    m->phases.push_back(dn);
    return MR_OK;
}

int reset_aux(mr_model *m);

// Buffers and the layer table of the work between steps (aux_step.cuh).
int setup_aux(mr_model *m) {
    const mr_model_config &c = m->cfg;
    m->aux_on = is_cbr(c) || is_lighting_memory(c);
    if (!m->aux_on) return MR_OK;
    MR_REQUIRE(m->ranks == 1, "chunk relays and latent memory run on one GPU");
    const int d = c.head_dim, h = c.hidden_size;
    int rc = MR_OK;
    auto falloc = [&](size_t n) { return static_cast<float *>(device_alloc(m, std::max<size_t>(n, 1) * 4, &rc)); };
    auto ialloc = [&](size_t n) { return static_cast<int *>(device_alloc(m, std::max<size_t>(n, 1) * 4, &rc)); };
    aux::Model &am = m->aux_model;
    am = aux::Model{};
    am.layers = c.layers;
    am.hidden = h;
    am.d = d;
    am.split_half = c.split_half_rope;
    am.norm_eps = c.norm_eps;
    am.inv_freq = m->d_inv_freq;
    am.lighting = is_lighting_memory(c) ? 1 : 0;
    am.chunk = c.cbr_chunk_size;
    am.slots = c.cbr_slots;
    am.memory_slots = c.memory_slots;
    am.latent = c.latent_dim;
    int *counts = ialloc(c.layers);
    if (rc) return rc;
    m->aux_host.assign(c.layers, aux::Layer{});
    m->aux_kvh = 0;
    for (int l = 0; l < c.layers && !rc; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        aux::Layer &L = m->aux_host[l];
        const TensorSlot *wk = tensor(m, p + "k"), *wv = tensor(m, p + "v"), *kn = tensor(m, p + "k_norm");
        MR_REQUIRE(wk && wv && kn && wk->dtype == wv->dtype, "layer %d: k / v / k_norm tensors", l);
        L.wk = wk->ptr;
        L.wv = wv->ptr;
        L.w_dt = wk->dtype;
        L.k_norm = kn->ptr;
        L.k_norm_dt = kn->dtype;
        L.kv_heads = m->layer_kvh[l];
        L.kv_width = L.kv_heads * d;
        m->aux_kvh = std::max(m->aux_kvh, L.kv_heads);
        L.relay_count = counts + l;
        L.last_pos = -1;
        L.stash_pos[0] = L.stash_pos[1] = -1;
        if (am.lighting) {
            const int cap = m->cache_capacity[l], ms = c.memory_slots, lat = c.latent_dim;
            MR_REQUIRE(lat <= 4096 && d <= 128, "latent memory: latent_dim %d / head_dim %d above 4096 / 128", lat, d);
            am.window = cap;
            const TensorSlot *ln = tensor(m, p + "latent_norm");
            MR_REQUIRE(ln, "layer %d: latent_norm", l);
            L.latent_norm = ln->ptr;
            L.latent_norm_dt = ln->dtype;
            L.lat_ring = falloc(static_cast<size_t>(cap) * lat);
            L.k_cache = m->k_cache[l];
            L.v_cache = m->v_cache[l];
            L.mem_lat = falloc(static_cast<size_t>(ms) * lat);
            L.mem_pos = ialloc(ms);
            L.mem_cnt = falloc(ms);
            L.mem_slot = ialloc(ms);
            L.stash_k = falloc(2 * static_cast<size_t>(L.kv_width));
            L.stash_v = falloc(2 * static_cast<size_t>(L.kv_width));
            L.stash_lat = falloc(2 * static_cast<size_t>(lat));
            L.relay_cap = ms;
        } else {
            const int C = c.cbr_chunk_size, S = c.cbr_slots;
            MR_REQUIRE(h <= 4096 && d <= 128, "chunk relays: hidden %d / head_dim %d above 4096 / 128", h, d);
            const TensorSlot *an = tensor(m, p + "a_norm"), *cbr = tensor(m, p + "cbr");
            MR_REQUIRE(an && cbr, "layer %d: a_norm / cbr", l);
            L.a_norm = an->ptr;
            L.a_norm_dt = an->dtype;
            L.pending = falloc(static_cast<size_t>(C) * h);
            float *q = falloc(static_cast<size_t>(S) * h);
            L.queries = q;
            L.u = falloc(static_cast<size_t>(C) * h);
            L.scores = falloc(static_cast<size_t>(S) * C);
            L.pooled = falloc(static_cast<size_t>(S) * h);
            L.anchors = falloc(S);
            L.relay_cap = (c.context_length / C) * S;
            if (rc) break;
            aux::k_norm_rows<<<S, 32, 0, m->ctx->stream>>>(cbr->ptr, cbr->dtype, S, h, c.cbr_norm_eps, q);
            MR_CUDA_TRY(cudaGetLastError());
        }
        L.relay_k = falloc(static_cast<size_t>(L.kv_heads) * std::max(1, L.relay_cap) * d);
        L.relay_v = falloc(static_cast<size_t>(L.kv_heads) * std::max(1, L.relay_cap) * d);
    }
    if (rc) return rc;
    m->aux_layers = static_cast<aux::Layer *>(device_alloc(m, sizeof(aux::Layer) * c.layers, &rc));
    if (rc) return rc;
    return reset_aux(m);
}

// A new sequence: the layer table as built (no relays, no memory, nothing planned).
int reset_aux(mr_model *m) {
    if (!m->aux_on) return MR_OK;
    MR_CUDA_TRY(cudaMemcpyAsync(m->aux_layers, m->aux_host.data(), sizeof(aux::Layer) * m->aux_host.size(),
                                cudaMemcpyHostToDevice, m->ctx->stream));
    MR_CUDA_TRY(cudaMemsetAsync(m->aux_host[0].relay_count, 0, sizeof(int) * m->aux_host.size(), m->ctx->stream));
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    return MR_OK;
}

// The work after one decode step (aux_step.cuh), queued behind it.
int launch_aux(mr_model *m) {
    cudaStream_t s = m->ctx->stream;
    const aux::Model &am = m->aux_model;
    const unsigned layers = static_cast<unsigned>(am.layers);
    aux::k_aux_plan<<<(am.layers + 127) / 128, 128, 0, s>>>(am, m->aux_layers, m->state);
    if (am.lighting) {
        aux::k_aux_merge<<<dim3(2, layers), aux::kThreads, 0, s>>>(am, m->aux_layers);
        aux::k_aux_move<<<dim3(8, layers), aux::kThreads, 0, s>>>(am, m->aux_layers);
        aux::k_aux_merged_kv<<<dim3(2 * m->aux_kvh, layers), aux::kThreads, 0, s>>>(am, m->aux_layers);
    } else {
        aux::k_cbr_scores<<<dim3(am.chunk, layers), aux::kThreads, 0, s>>>(am, m->aux_layers);
        aux::k_cbr_pool<<<dim3(am.slots, layers), aux::kThreads, sizeof(float) * am.chunk, s>>>(am, m->aux_layers,
                                                                                               m->state);
        aux::k_cbr_kv<<<dim3(am.slots * 2 * m->aux_kvh, layers), aux::kThreads, 0, s>>>(am, m->aux_layers);
    }
    MR_CUDA_TRY(cudaGetLastError());
    return MR_OK;
}

int build_plan(mr_model *m) {
    const mr_model_config &c = m->cfg;
    if (!is_engine_family(c))
        return set_error(MR_ERR_ARGUMENT, "family %d is not supported by this engine build yet", c.family);
    m->phases.clear();
    const TensorSlot *embed = tensor(m, "embed");
    for (int l = 0; l < c.layers; ++l) {
        if (is_lighting(c)) {
            if (int rc = plan_lighting_layer(m, l)) return rc;
            continue;
        }
        const std::string p = "layers." + std::to_string(l) + ".";
        // 1. RMSNorm(x) -> q, k, v (layer 0 reads the embedding row directly)
        Phase qkv = gemv_phase(l, m->x, tensor(m, p + "a_norm"), c.norm_eps);
        if (l == 0) {
            qkv.gemv.input_kind = IN_EMBED_ROW;
            qkv.gemv.embed = embed->ptr;
            qkv.gemv.embed_dtype = embed->dtype;
        }
        qkv.gemv.nseg = 3;
        qkv.gemv.seg[0] = segment(tensor(m, p + "q"), m->q_raw);
        qkv.gemv.seg[1] = segment(tensor(m, p + "k"), m->k_raw);
        qkv.gemv.seg[2] = segment(tensor(m, p + "v"), m->v_raw);
        qkv.gemv.epilogue = EPI_STORE;
        qkv.gemv.skip = m->xres_skip;
        if (is_cbr(c)) {  // the chunk's layer inputs, pooled into relays between steps
            qkv.gemv.save_in = m->aux_host[l].pending;
            qkv.gemv.save_rows = c.cbr_chunk_size;
        }
        m->phases.push_back(qkv);
        // 2. attention (flashnano-1.6: the ring, then the relay rows)
        Phase at{};
        if (int rc = attn_phase(m, l, c.qk_norm, 1, at)) return rc;
        if (is_cbr(c)) {
            at.attn.relay_k = m->aux_host[l].relay_k;
            at.attn.relay_v = m->aux_host[l].relay_v;
            at.attn.relay_count = m->aux_host[l].relay_count;
            at.attn.relay_capacity = m->aux_host[l].relay_cap;
        }
        m->phases.push_back(at);
        // 3. o projection of the attention output + residual (model.py:282)
        Phase o = gemv_phase(l, m->attn_out, nullptr, 0.f);
        o.gemv.nseg = 1;
        o.gemv.seg[0] = segment(tensor(m, p + "o"));
        o.gemv.epilogue = EPI_RESIDUAL;
        o.gemv.scale = c.residual_scale;
        o.gemv.x = m->x;
        o.gemv.skip = m->xres_skip;
        m->phases.push_back(o);
        // 4. RMSNorm(x) -> gate, up -> SwiGLU (model.py:87-89)
        Phase gu = gemv_phase(l, m->x, tensor(m, p + "f_norm"), c.norm_eps);
        gu.gemv.nseg = 2;
        gu.gemv.seg[0] = segment(tensor(m, p + "ffn.gate"));
        gu.gemv.seg[1] = segment(tensor(m, p + "ffn.up"));
        gu.gemv.epilogue = EPI_SWIGLU;
        gu.gemv.out = m->ffn;
        m->phases.push_back(gu);
        // 5. down projection + residual (model.py:283)
        Phase dn = gemv_phase(l, m->ffn, nullptr, 0.f);
        dn.gemv.nseg = 1;
        dn.gemv.seg[0] = segment(tensor(m, p + "ffn.down"));
        dn.gemv.epilogue = EPI_RESIDUAL;
        dn.gemv.scale = c.residual_scale;
        dn.gemv.x = m->x;
        dn.gemv.skip = m->xres_skip;
        m->phases.push_back(dn);
    }
    // final RMSNorm + head (model.py:285, 307)
    Phase head = gemv_phase(-1, m->x, tensor(m, "norm"), c.norm_eps);
    head.gemv.nseg = 1;
    head.gemv.seg[0] = segment(tensor(m, c.tie_embeddings ? "embed" : "output"));
    head.gemv.epilogue = EPI_LOGITS;
    head.gemv.logits = m->logits;
    m->phases.push_back(head);
    Phase end{};
    end.kind = PH_STEP_END;
    end.layer = -2;
    m->phases.push_back(end);
    // Tensor parallel: each rank computes a contiguous slice of every segment's
    // rows (the o / down slices are its residual rows) and of the KV heads.
    for (Phase &ph : m->phases) {
        if (ph.kind == PH_GEMV) {
            for (int i = 0; i < ph.gemv.nseg; ++i)
                rank_rows(ph.gemv.seg[i].rows, m->rank, m->ranks, ph.gemv.seg[i].row_lo, ph.gemv.seg[i].row_n);
        } else if (ph.kind == PH_ATTN_GQA) {
            rank_rows(ph.attn.kv_heads, m->rank, m->ranks, ph.attn.kv_lo, ph.attn.kv_n);
        }
    }
    // Weight streaming through the shared-memory ring: pieces of whole 16-byte
    // rows (cp.async.bulk granularity) within the phase's piece cap.
    for (Phase &ph : m->phases) {
        if (ph.kind != PH_GEMV) continue;
        GemvPhase &g = ph.gemv;
        int piece_cap, group_cap;
        phase_caps(m, g, piece_cap, group_cap);
        bool bulk = true;
        for (int i = 0; i < g.nseg; ++i) {
            const int row_bytes = g.seg[i].cols * (int)dtype_size(g.seg[i].dtype);
            if (row_bytes % 16 || row_bytes > piece_cap) bulk = false;
            // a SwiGLU gate/up pair shares one group of at most kRowBatch rows
            else g.seg[i].rows_per_piece = std::max(1, std::min(g.epilogue == EPI_SWIGLU ? kRowBatch / 2 : kRowBatch,
                                                                piece_cap / row_bytes));
        }
        if (g.epilogue == EPI_SWIGLU && g.seg[0].rows_per_piece != g.seg[1].rows_per_piece) bulk = false;
        g.bulk = bulk;
        g.wdtype = g.seg[0].dtype;
        for (int i = 1; i < g.nseg; ++i)
            if (g.seg[i].dtype != g.wdtype) g.wdtype = -1;
        // the input vector is staged split only where the ring feeds 16-bit rows of one dtype
        g.xsplit = bulk && (g.wdtype == MR_DTYPE_BF16 || g.wdtype == MR_DTYPE_F16);
        const int gain_bytes = (g.seg[0].cols * (int)dtype_size(g.norm_gain_dtype) + 15) & ~15;
        g.gain_piece = bulk && g.norm && g.norm_gain && gain_bytes <= piece_cap;
    }
    return MR_OK;
}

// Whether CTA b owns any rows of the phase (a CTA with none skips the phase).
bool cta_has_rows(const GemvPhase &g, int b, int G) {
    for (int s = 0; s < g.nseg; ++s) {
        int r0, r1;
        seg_cta_rows(g.seg[s], b, G, g.skip, r0, r1);
        if (r1 > r0) return true;
    }
    return false;
}

// The weight stream of every CTA: its pieces of every bulk phase, in the
// order the kernel consumes them (gain vector first, then the rows; SwiGLU
// phases alternate gate and up pieces of the same rows).
int build_pieces(mr_model *m) {
    const int G = m->grid;
    std::vector<std::vector<PieceDesc>> per(G);
    for (size_t p = 0; p < m->phases.size(); ++p) {
        const Phase &ph = m->phases[p];
        if (ph.kind != PH_GEMV || !ph.gemv.bulk) continue;
        const GemvPhase &g = ph.gemv;
        const uint32_t gain_bytes = (uint32_t)((g.seg[0].cols * (int)dtype_size(g.norm_gain_dtype) + 15) & ~15);
        auto add = [&](std::vector<PieceDesc> &v, int s, int row0, int n) {
            const Segment &seg = g.seg[s];
            const size_t row_bytes = (size_t)seg.cols * dtype_size(seg.dtype);
            PieceDesc d{};
            d.src = static_cast<const char *>(seg.w) + row_bytes * row0;
            d.bytes = (uint32_t)(row_bytes * n);
            d.phase = (int)p;
            v.push_back(d);
        };
        for (int b = 0; b < G; ++b) {
            std::vector<PieceDesc> &v = per[b];
            if (g.gain_piece && cta_has_rows(g, b, G)) {
                PieceDesc d{};
                d.src = g.norm_gain;
                d.bytes = gain_bytes;
                d.phase = (int)p;
                v.push_back(d);
            }
            const bool paired = g.epilogue == EPI_SWIGLU;
            for (int s = 0; s < (paired ? 1 : g.nseg); ++s) {
                const int rpp = g.seg[s].rows_per_piece;
                int r0, r1;
                seg_cta_rows(g.seg[s], b, G, g.skip, r0, r1);
                for (int row0 = r0; row0 < r1; row0 += rpp) {
                    const int n = std::min(rpp, r1 - row0);
                    add(v, s, row0, n);
                    if (paired) add(v, 1, row0, n);
                }
            }
        }
    }
    size_t stride = 1;
    for (auto &v : per) stride = std::max(stride, v.size());
    std::vector<PieceDesc> flat(stride * G);
    std::vector<int> counts(G);
    for (int b = 0; b < G; ++b) {
        std::copy(per[b].begin(), per[b].end(), flat.begin() + (size_t)b * stride);
        counts[b] = (int)per[b].size();
    }
    int rc = MR_OK;
    m->d_pieces = static_cast<PieceDesc *>(device_alloc(m, sizeof(PieceDesc) * flat.size(), &rc));
    m->d_piece_count = static_cast<int *>(device_alloc(m, sizeof(int) * G, &rc));
    if (rc) return rc;
    MR_CUDA_TRY(cudaMemcpy(m->d_pieces, flat.data(), sizeof(PieceDesc) * flat.size(), cudaMemcpyHostToDevice));
    MR_CUDA_TRY(cudaMemcpy(m->d_piece_count, counts.data(), sizeof(int) * G, cudaMemcpyHostToDevice));
    m->piece_stride = (int)stride;
    return MR_OK;
}

// Piece groups of every (bulk phase, CTA), in the stream order of
// build_pieces: greedy, a group closes before the piece (or gate/up pair) that
// would take its rows past the phase's group cap, kRowBatch rows or kGroupPieces
// pieces.
int build_groups(mr_model *m) {
    const int G = m->grid;
    std::vector<GroupTable> flat;
    for (Phase &ph : m->phases) {
        if (ph.kind != PH_GEMV || !ph.gemv.bulk) continue;
        GemvPhase &g = ph.gemv;
        int piece_cap, cap;
        phase_caps(m, g, piece_cap, cap);
        const bool paired = g.epilogue == EPI_SWIGLU;
        const int cols = g.seg[0].cols, per = paired ? 2 : 1;
        std::vector<std::vector<GroupTable>> per_cta(G);
        size_t stride = 1;
        for (int b = 0; b < G; ++b) {
            std::vector<GroupTable> &out = per_cta[b];
            GroupTable t{};
            int bytes = 0;
            auto close = [&]() {
                out.push_back(t);
                t = GroupTable{};
                bytes = 0;
            };
            // The gain vector (at most a quarter of the ring) rides in the first
            // group without counting against the half-ring cap: a group still
            // spans at most three quarters of the ring, which it always finds
            // once the older pieces are released (a wrap wastes less than one
            // piece, at most a quarter).  Counting it split the first group
            // of CTAs whose rows just fill half the ring.
            if (g.gain_piece && cta_has_rows(g, b, G)) {
                t.p[0] = GroupPiece{-1, 0, 0, 0};
                t.count = 1;
            }
            for (int s = 0; s < (paired ? 1 : g.nseg); ++s) {
                const int rpp = g.seg[s].rows_per_piece;
                int r0, r1;
                seg_cta_rows(g.seg[s], b, G, g.skip, r0, r1);
                for (int row0 = r0; row0 < r1; row0 += rpp) {
                    const int n = std::min(rpp, r1 - row0);
                    int ubytes = n * cols * (int)dtype_size(g.seg[s].dtype);
                    if (paired) ubytes += n * cols * (int)dtype_size(g.seg[s + 1].dtype);
                    if (t.count > 0 &&
                        (bytes + ubytes > cap || t.rows + per * n > kRowBatch || t.count + per > kGroupPieces))
                        close();
                    t.p[t.count++] = GroupPiece{s, row0, n, t.rows};
                    t.rows += n;
                    if (paired) {
                        t.p[t.count++] = GroupPiece{s + 1, row0, n, t.rows};
                        t.rows += n;
                    }
                    bytes += ubytes;
                }
            }
            out.push_back(t);
            for (size_t k = 0; k + 1 < out.size(); ++k) out[k].more = 1;
            stride = std::max(stride, out.size());
        }
        g.group_offset = (int)flat.size();
        g.group_stride = (int)stride;
        for (int b = 0; b < G; ++b)
            for (size_t k = 0; k < stride; ++k) flat.push_back(k < per_cta[b].size() ? per_cta[b][k] : GroupTable{});
    }
    for (size_t p = 0; p < m->phases.size(); ++p) {
        Phase &ph = m->phases[p];
        ph.next_groups = -1;
        ph.next_group_stride = 0;
        if (p + 1 < m->phases.size() && m->phases[p + 1].kind == PH_GEMV && m->phases[p + 1].gemv.bulk) {
            ph.next_groups = m->phases[p + 1].gemv.group_offset;
            ph.next_group_stride = m->phases[p + 1].gemv.group_stride;
        }
    }
    if (flat.empty()) flat.push_back(GroupTable{});
    int rc = MR_OK;
    m->d_groups = static_cast<GroupTable *>(device_alloc(m, sizeof(GroupTable) * flat.size(), &rc));
    if (rc) return rc;
    MR_CUDA_TRY(cudaMemcpy(m->d_groups, flat.data(), sizeof(GroupTable) * flat.size(), cudaMemcpyHostToDevice));
    return MR_OK;
}

// The device step's error word -> a status (and the latched failure).
int error_status(mr_model *m, int error, const char *what) {
    if (!error) return MR_OK;
    m->failed = true;
    if (error == 3) return set_error(MR_ERR_STATE, "%s: context_length exceeded on the device", what);
    if (error == 4) return set_error(MR_ERR_STATE, "%s: a token outside the vocabulary reached the device", what);
    return set_error(MR_ERR_TIMEOUT, "%s: device wait timed out (code %d); call reset()", what, error);
}

int sync_and_check(mr_model *m, const char *what) {
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    int error = 0;
    MR_CUDA_TRY(cudaMemcpy(&error, &m->state->error, sizeof(int), cudaMemcpyDeviceToHost));
    return error_status(m, error, what);
}

int ensure_feed(mr_model *m, int n) {
    if (n <= m->feed_capacity) return MR_OK;
    int rc = MR_OK;
    const int cap = std::max(n, 256);
    m->feed = static_cast<int *>(device_alloc(m, sizeof(int) * cap, &rc));
    if (rc) return rc;
    m->feed_capacity = cap;
    return MR_OK;
}

int ensure_gen(mr_model *m, int n) {
    if (n <= m->gen_capacity) return MR_OK;
    int rc = MR_OK;
    const int cap = std::max(n, 256);
    m->gen_out = static_cast<int *>(device_alloc(m, sizeof(int) * cap, &rc));
    if (rc) return rc;
    m->gen_capacity = cap;
    return MR_OK;
}

int launch_step(mr_model *m, const StepControl &ctl) {
    int nphases = (int)m->phases.size();
    StepControl control = ctl;
    // distinct exchange tags per launch (tags repeat only after 2^32 / nphases launches)
    control.tag_base = static_cast<unsigned int>(++m->launches * static_cast<unsigned long long>(nphases));
    void *args[] = {&m->d_phases, &nphases, &m->state, &control};
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(m->grid);
    cfg.blockDim = dim3(kBlockThreads);
    cfg.dynamicSmemBytes = m->smem_bytes;
    cfg.stream = m->ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MR_CUDA_TRY(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void *>(decode_step_kernel), args));
    return m->aux_on ? launch_aux(m) : MR_OK;
}

StepControl base_control(mr_model *m) {
    StepControl ctl{};
    ctl.withhold_phase = m->withhold_phase;
    ctl.feed = m->feed;
    ctl.feed_base = m->position;
    ctl.logits_rows = m->logits_rows;
    ctl.eos = -1;
    ctl.context_length = m->cfg.context_length;
    ctl.vocab_size = m->cfg.vocab_size;
    ctl.scratch_floats = m->scratch_floats;
    ctl.attn_base = m->attn_base;
    ctl.inv_freq = m->d_inv_freq;
    ctl.rope_pairs = m->cfg.head_dim / 2;
    const TensorSlot *embed = tensor(m, "embed");
    ctl.embed = embed->ptr;
    ctl.embed_dtype = embed->dtype;
    ctl.hidden = m->cfg.hidden_size;
    ctl.xres_skip = m->xres_skip;
    ctl.xres_lo = m->xres_lo;
    ctl.xres_n = m->xres_n;
    ctl.ranks = m->ranks;
    ctl.rank = m->rank;
    ctl.arena = m->arena;
    for (int j = 0; j < m->ranks; ++j) ctl.peers[j] = m->peer[j];
    ctl.best_slots = m->best_slots;
    ctl.ring_bytes = m->ring_bytes;
    ctl.pieces = m->d_pieces;
    ctl.groups = m->d_groups;
    ctl.piece_count = m->d_piece_count;
    ctl.piece_stride = m->piece_stride;
    return ctl;
}

int ready(mr_model *m) {
    MR_REQUIRE(m, "model is NULL");
    if (!m->finalized) return set_error(MR_ERR_STATE, "model is not finalized");
    if (m->op_path)
        return set_error(MR_ERR_STATE, "family %d has no decode-engine plan: its token step runs on the host over "
                         "the op kernels (mr_model_linear and mr_op_*)", m->cfg.family);
    if (m->failed)
        return set_error(MR_ERR_STATE, "A previous device operation failed; call reset() before reusing this model");
    if (m->ranks > 1 && !m->connected)
        return set_error(MR_ERR_STATE, "tensor-parallel model: mr_model_tp_connect has not been called");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    return MR_OK;
}

int host_argmax(const float *v, int n) {  // numpy.argmax: the first maximum
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (v[i] > v[best]) best = i;
    return best;
}

// heavy-medium-2.0: n tokens through the device token step; the logits of
// every token (return_all) or of the last one are copied to `out`.
constexpr int kHeavyChunk = 4096;  // tokens per Heavy Medium batched chunk
int heavy_feed(mr_model *m, const int *ids, int n, int return_all, float *out) {
    const int V = m->cfg.vocab_size;
    for (int i = 0; i < n; ++i) MR_REQUIRE(ids[i] >= 0 && ids[i] < V, "input token is outside the vocabulary");
    MR_REQUIRE(m->position + n <= m->cfg.context_length,
               "input would exceed context_length; reset or allocate a larger context");
    // a prompt of several tokens: batched chunks (GEMMs on tcgen05), else the token step
    int first = 0;
    if (n > 1 && m->prefill_on && heavy_batchable(m->heavy)) {
        for (; first < n;) {
            const int T = std::min(kHeavyChunk, n - first);
            int rc = heavy_prefill(m->heavy, ids + first, T, m->position, return_all != 0);
            if (!rc && out && (return_all || first + T == n)) {
                const size_t rows = return_all ? T : 1;
                const cudaError_t err =
                    cudaMemcpyAsync(out + (return_all ? static_cast<size_t>(first) * V : 0), heavy_prefill_logits(m->heavy),
                                    sizeof(float) * V * rows, cudaMemcpyDeviceToHost, m->ctx->stream);
                if (err != cudaSuccess) rc = cuda_error(err, "logits read");
            }
            if (rc) {
                m->failed = true;
                return rc;
            }
            m->position += T;
            first += T;
        }
    }
    for (int i = first; i < n; ++i) {
        int rc = heavy_token(m->heavy, ids[i], m->position);
        if (!rc && out && (return_all || i == n - 1)) {
            const cudaError_t err = cudaMemcpyAsync(out + (return_all ? (size_t)i * V : 0), heavy_logits(m->heavy),
                                                    sizeof(float) * V, cudaMemcpyDeviceToHost, m->ctx->stream);
            if (err != cudaSuccess) rc = cuda_error(err, "logits read");
        }
        if (rc) {
            m->failed = true;
            return rc;
        }
        ++m->position;
    }
    const cudaError_t err = cudaStreamSynchronize(m->ctx->stream);
    if (err != cudaSuccess) {
        m->failed = true;
        return cuda_error(err, "heavy-medium-2.0 token step");
    }
    const int rc = heavy_status(m->heavy);  // a bounded device wait that gave up
    if (rc) m->failed = true;
    return rc;
}

// Runs n fed tokens starting at the current position; logits of the selected
// rows are copied to `out` (return_all: n rows, else the last row only).
constexpr int kPrefillChunk = 512;  // tokens per batched prefill chunk

// The batched prefill applies when every projection and the lm_head are BF16
// and the widths are whole 16-byte rows; otherwise prompts run token by token
// through the decode kernel.
void setup_prefill(mr_model *m) {
    const mr_model_config &c = m->cfg;
    const int d = c.head_dim, q = c.query_heads * d;
    m->prefill_ok = false;
    const bool lighting = is_lighting_ring(c);
    if (!is_gqa_family(c.family) && !lighting) return;
    const int gq_max = c.query_heads / *std::min_element(m->layer_kvh.begin(), m->layer_kvh.end());
    if (c.hidden_size % 8 || q % 8 || c.ffn_dim % 8 || d % 4 || gq_max > 32) return;
    if (lighting && c.latent_dim % 8) return;
    auto bf16 = [&](const std::string &name) {
        const TensorSlot *t = tensor(m, name);
        return t && t->dtype == MR_DTYPE_BF16 ? t->ptr : nullptr;
    };
    PrefillModel &pm = m->pm;
    pm.stream = m->ctx->stream;
    pm.hidden = c.hidden_size;
    pm.heads = c.query_heads;
    pm.head_dim = d;
    pm.ffn = c.ffn_dim;
    pm.vocab = c.vocab_size;
    pm.kv_max = *std::max_element(m->layer_kvh.begin(), m->layer_kvh.end());
    pm.eps = c.norm_eps;
    pm.residual_scale = c.residual_scale;
    pm.qk_norm = lighting ? 1 : c.qk_norm;
    pm.split_half = c.split_half_rope;
    pm.lighting = lighting;
    pm.latent_dim = c.latent_dim;
    const TensorSlot *embed = tensor(m, "embed"), *norm = tensor(m, "norm");
    pm.embed = embed->ptr;
    pm.embed_dt = embed->dtype;
    pm.final_norm = norm->ptr;
    pm.final_norm_dt = norm->dtype;
    pm.head = bf16(c.tie_embeddings ? "embed" : "output");
    pm.inv_freq = m->d_inv_freq;
    if (!pm.head) return;
    pm.layers.clear();
    for (int l = 0; l < c.layers; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        PrefillLayer L{};
        const TensorSlot *an = tensor(m, p + "a_norm");
        L.a_norm = an->ptr;
        L.a_norm_dt = an->dtype;
        if (!lighting) {
            const TensorSlot *fn = tensor(m, p + "f_norm");
            L.f_norm = fn->ptr;
            L.f_norm_dt = fn->dtype;
        } else {
            const TensorSlot *ln = tensor(m, p + "latent_norm");
            L.latent_norm = ln->ptr;
            L.latent_norm_dt = ln->dtype;
            L.latent = bf16(p + "latent");
            float ag = 0.f, fg = 0.f;
            if (read_scalar(m, p + "attention_gate", ag) || read_scalar(m, p + "ffn_gate", fg) || !L.latent) return;
            L.o_scale = c.residual_scale * ag;
            L.down_scale = c.residual_scale * fg;
        }
        if (c.qk_norm || lighting) {
            const TensorSlot *qn = tensor(m, p + "q_norm"), *kn = tensor(m, p + "k_norm");
            L.q_norm = qn->ptr;
            L.k_norm = kn->ptr;
            L.qk_norm_dt = qn->dtype;
        }
        L.q = bf16(p + "q");
        L.k = bf16(p + "k");
        L.v = bf16(p + "v");
        L.o = bf16(p + "o");
        L.gate = bf16(p + "ffn.gate");
        L.up = bf16(p + "ffn.up");
        L.down = bf16(p + "ffn.down");
        if (!L.q || !L.k || !L.v || !L.o || !L.gate || !L.up || !L.down) return;
        L.k_cache = m->k_cache[l];
        L.v_cache = m->v_cache[l];
        L.capacity = m->cache_capacity[l];
        L.kv_heads = m->layer_kvh[l];
        pm.layers.push_back(L);
    }
    m->prefill_ok = true;
}

// Batched prefill: chunks of up to kPrefillChunk tokens through prefill_chunk,
// then the device step state moves to the new position.
int run_feed_batched(mr_model *m, int n, int return_all, float *out) {
    const int V = m->cfg.vocab_size;
    cudaStream_t st = m->ctx->stream;
    int rc = prefill_reserve(m->pm, m->pw, std::min(n, kPrefillChunk), return_all != 0);
    if (rc) return rc;
    for (int done = 0; done < n;) {
        const int T = std::min(kPrefillChunk, n - done);
        rc = prefill_chunk(m->pm, m->pw, m->feed + done, T, m->position + done, return_all != 0);
        if (rc) {
            m->failed = true;
            return rc;
        }
        if (return_all && out)
            MR_CUDA_TRY(cudaMemcpyAsync(out + (size_t)done * V, m->pw.logits, sizeof(float) * (size_t)T * V,
                                        cudaMemcpyDeviceToHost, st));
        done += T;
    }
    if (!return_all && out) MR_CUDA_TRY(cudaMemcpyAsync(out, m->pw.logits, sizeof(float) * V, cudaMemcpyDeviceToHost, st));
    const int position = m->position + n;
    MR_CUDA_TRY(cudaMemcpyAsync(&m->state->position, &position, sizeof(int), cudaMemcpyHostToDevice, st));
    cudaError_t err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) {
        m->failed = true;
        return cuda_error(err, "batched prefill");
    }
    rc = prefill_status(m->pm, m->pw);
    if (rc) {
        m->failed = true;
        return rc;
    }
    m->position = position;
    return MR_OK;
}

// Decode calls (a few tokens, last logits only) through page-locked staging:
// ids in, n launches, then the error word and the logits out, one synchronise.
int run_feed_staged(mr_model *m, const int *ids, int n, float *out) {
    cudaStream_t st = m->ctx->stream;
    const int V = m->cfg.vocab_size;
    memcpy(m->h_ids, ids, sizeof(int) * n);
    MR_CUDA_TRY(cudaMemcpyAsync(m->feed, m->h_ids, sizeof(int) * n, cudaMemcpyHostToDevice, st));
    StepControl ctl = base_control(m);
    ctl.feed_len = n;
    for (int i = 0; i < n; ++i) {
        const int rc = launch_step(m, ctl);
        if (rc) {
            m->failed = true;
            return rc;
        }
    }
    MR_CUDA_TRY(cudaMemcpyAsync(m->h_error, &m->state->error, sizeof(int), cudaMemcpyDeviceToHost, st));
    if (out) MR_CUDA_TRY(cudaMemcpyAsync(m->h_logits, m->logits, sizeof(float) * V, cudaMemcpyDeviceToHost, st));
    MR_CUDA_TRY(cudaStreamSynchronize(st));
    if (const int rc = error_status(m, *m->h_error, "decode")) return rc;
    if (out) memcpy(out, m->h_logits, sizeof(float) * V);
    m->position += n;
    return MR_OK;
}

int run_feed(mr_model *m, const int *ids, int n, int return_all, float *out) {
    const int V = m->cfg.vocab_size;
    for (int i = 0; i < n; ++i) MR_REQUIRE(ids[i] >= 0 && ids[i] < V, "input token is outside the vocabulary");
    MR_REQUIRE(m->position + n <= m->cfg.context_length,
               "input would exceed context_length; reset or allocate a larger context");
    int rc = ensure_feed(m, n);
    if (rc) return rc;
    if (!return_all && n <= mr_model::kHostIds && m->h_ids && !(m->prefill_ok && m->prefill_on && n > 1))
        return run_feed_staged(m, ids, n, out);
    MR_CUDA_TRY(cudaMemcpyAsync(m->feed, ids, sizeof(int) * n, cudaMemcpyHostToDevice, m->ctx->stream));
    if (m->prefill_ok && m->prefill_on && n > 1) return run_feed_batched(m, n, return_all, out);
    StepControl ctl = base_control(m);
    ctl.feed_len = n;
    ctl.return_all = return_all;
    int done = 0;
    while (done < n) {
        const int batch = return_all ? std::min(m->logits_rows, n - done) : n - done;
        for (int i = 0; i < batch; ++i) {
            rc = launch_step(m, ctl);
            if (rc) {
                m->failed = true;
                return rc;
            }
        }
        if (return_all && out) {
            for (int i = 0; i < batch; ++i) {
                const int row = (done + i) % m->logits_rows;
                MR_CUDA_TRY(cudaMemcpyAsync(out + (size_t)(done + i) * V, m->logits + (size_t)row * V,
                                            sizeof(float) * V, cudaMemcpyDeviceToHost, m->ctx->stream));
            }
        }
        rc = sync_and_check(m, "prefill");
        if (rc) return rc;
        done += batch;
    }
    if (!return_all && out) MR_CUDA_TRY(cudaMemcpy(out, m->logits, sizeof(float) * V, cudaMemcpyDeviceToHost));
    m->position += n;
    return MR_OK;
}

}  // namespace

namespace mr {
// A finalized model's resident tensor (tensor_ops.cu): device pointer, stored
// dtype, and its shape as rows x cols (1-D tensors: 1 x n).
int model_tensor(mr_model *m, const char *name, const void **ptr, int *dtype, int64_t *rows, int64_t *cols) {
    MR_REQUIRE(m && name, "NULL argument");
    if (!m->finalized) return set_error(MR_ERR_STATE, "model is not finalized");
    auto it = m->tensors.find(name);
    MR_REQUIRE(it != m->tensors.end(), "unknown tensor %s", name);
    const TensorSlot &t = it->second;
    *ptr = t.ptr;
    *dtype = t.dtype;
    *rows = t.shape.size() == 2 ? t.shape[0] : 1;
    *cols = t.shape.size() == 2 ? t.shape[1] : t.shape[0];
    return MR_OK;
}
int model_stream(mr_model *m, cudaStream_t *stream, int *device) {
    MR_REQUIRE(m, "model is NULL");
    *stream = m->ctx->stream;
    *device = m->ctx->device;
    return MR_OK;
}
}  // namespace mr

extern "C" {

int mr_model_create(mr_context *ctx, const mr_model_config *config, const int *layer_kv_heads,
                    const int *layer_window, const float *inv_freq, mr_model **out) {
    MR_REQUIRE(ctx && config && layer_kv_heads && layer_window && inv_freq && out, "NULL argument");
    const mr_model_config &c = *config;
    MR_REQUIRE(c.family >= 0 && c.family <= MR_FAMILY_HEAVY_MEDIUM_20, "unknown family %d", c.family);
    MR_REQUIRE(c.vocab_size > 0 && c.hidden_size > 0 && c.layers > 0 && c.query_heads > 0 && c.kv_heads > 0 &&
                   c.head_dim > 0 && c.head_dim % 2 == 0 && c.ffn_dim > 0 && c.context_length > 0,
               "invalid model geometry");
    MR_REQUIRE(c.head_dim <= 256, "head_dim %d too large for the engine", c.head_dim);
    for (int l = 0; l < c.layers; ++l)
        MR_REQUIRE(layer_kv_heads[l] > 0 && c.query_heads % layer_kv_heads[l] == 0, "layer %d: invalid KV head count",
                   l);
    MR_CUDA_TRY(cudaSetDevice(ctx->device));
    auto *m = new mr_model();
    mr::context_retain(ctx);
    m->ctx = ctx;
    m->cfg = c;
    m->layer_kvh.assign(layer_kv_heads, layer_kv_heads + c.layers);
    m->layer_window.assign(layer_window, layer_window + c.layers);
    m->inv_freq.assign(inv_freq, inv_freq + c.head_dim / 2);
    expected_tensors(m);
    m->grid = ctx->sm_count;
    *out = m;
    return MR_OK;
}

int mr_model_destroy(mr_model *m) {
    if (!m) return MR_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    for (int j = 0; j < kMaxRanks; ++j)
        if (m->peer_open[j]) cudaIpcCloseMemHandle(m->peer[j]);
    for (void *p : m->allocations) cudaFree(p);
    prefill_release(m->pw);
    heavy_destroy(m->heavy);
    sampler_destroy(m->sampler);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->h_ids) cudaFreeHost(m->h_ids);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->ev1) cudaEventDestroy(m->ev1);
    for (int i = 0; i < 2; ++i) {
        if (m->staging[i]) cudaFreeHost(m->staging[i]);
        if (m->staged[i]) cudaEventDestroy(m->staged[i]);
    }
    mr_context *ctx = m->ctx;
    delete m;
    mr::context_release(ctx);
    return MR_OK;
}

int mr_model_load_tensor(mr_model *m, const char *name, int dtype, int ndim, const int64_t *shape,
                         const void *host) {
    MR_REQUIRE(m && host, "NULL argument");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    TensorSlot *t = nullptr;
    int rc = check_tensor(m, name, dtype, ndim, shape, &t);
    if (rc) return rc;
    MR_CUDA_TRY(cudaMemcpyAsync(t->ptr, host, t->bytes, cudaMemcpyHostToDevice, m->ctx->stream));
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    return MR_OK;
}

namespace {
constexpr size_t kStagingBytes = size_t(64) << 20;

// Closes a file descriptor on every return path.
struct FileHandle {
    int fd = -1;
    ~FileHandle() {
        if (fd >= 0) close(fd);
    }
};
}  // namespace

int mr_model_load_file(mr_model *m, const char *name, int dtype, int ndim, const int64_t *shape, const char *path,
                       uint64_t offset) {
    MR_REQUIRE(m && path, "NULL argument");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    TensorSlot *t = nullptr;
    int rc = check_tensor(m, name, dtype, ndim, shape, &t);
    if (rc) return rc;
    for (int i = 0; i < 2; ++i) {
        if (!m->staging[i]) MR_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&m->staging[i]), kStagingBytes,
                                                      cudaHostAllocDefault));
        if (!m->staged[i]) MR_CUDA_TRY(cudaEventCreateWithFlags(&m->staged[i], cudaEventDisableTiming));
    }
    FileHandle file;
    file.fd = open(path, O_RDONLY | O_CLOEXEC);
    MR_REQUIRE(file.fd >= 0, "%s: cannot open %s", name, path);
    posix_fadvise(file.fd, static_cast<off_t>(offset), static_cast<off_t>(t->bytes), POSIX_FADV_SEQUENTIAL);
    // chunk i is read into buffer i % 2 while chunk i - 1 is copied to HBM from the other one
    size_t done = 0;
    for (int i = 0; done < t->bytes; ++i) {
        const int b = i & 1;
        const size_t n = std::min(kStagingBytes, t->bytes - done);
        MR_CUDA_TRY(cudaEventSynchronize(m->staged[b]));  // the copy out of this buffer (chunk i - 2) is done
        for (size_t got = 0; got < n;) {
            const ssize_t r = pread(file.fd, m->staging[b] + got, n - got, static_cast<off_t>(offset + done + got));
            MR_REQUIRE(r > 0, "%s: %s ends before the tensor's %zu bytes at offset %llu", name, path, t->bytes,
                       static_cast<unsigned long long>(offset));
            got += static_cast<size_t>(r);
        }
        MR_CUDA_TRY(cudaMemcpyAsync(static_cast<unsigned char *>(t->ptr) + done, m->staging[b], n,
                                    cudaMemcpyHostToDevice, m->ctx->stream));
        MR_CUDA_TRY(cudaEventRecord(m->staged[b], m->ctx->stream));
        done += n;
    }
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    return MR_OK;
}

int mr_model_fill_synthetic(mr_model *m, const char *name, int dtype, int ndim, const int64_t *shape,
                            uint64_t seed, int tensor_index, float scale, float fill) {
    MR_REQUIRE(m, "NULL argument");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    TensorSlot *t = nullptr;
    int rc = check_tensor(m, name, dtype, ndim, shape, &t);
    if (rc) return rc;
    const size_t n = t->bytes / dtype_size(dtype);
    const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 64);
    if (scale != 0.0f) {
        MR_REQUIRE(dtype == MR_DTYPE_BF16, "%s: the hash generator produces BF16 only", name);
        const uint64_t key = host_splitmix(seed * 0x9E3779B97F4A7C15ull + (uint64_t)(tensor_index + 1));
        k_fill_hash_bf16<<<blocks, 256, 0, m->ctx->stream>>>(static_cast<uint16_t *>(t->ptr), n, key, scale);
    } else {
        k_fill_value<<<blocks, 256, 0, m->ctx->stream>>>(t->ptr, dtype, n, fill);
    }
    MR_CUDA_TRY(cudaGetLastError());
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    return MR_OK;
}

int mr_model_finalize(mr_model *m) {
    MR_REQUIRE(m, "model is NULL");
    MR_REQUIRE(!m->finalized, "model already finalized");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    for (auto &kv : m->tensors)
        if (!kv.second.ptr || kv.second.dtype < 0)
            return set_error(MR_ERR_ARGUMENT, "Missing tensor %s", kv.first.c_str());
    if (m->cfg.family == MR_FAMILY_HEAVY_MEDIUM_20) {
        m->finalized = true;  // the tensors are complete: heavy_create reads them by name
        const int rc = heavy_create(m, m->cfg, m->ctx->stream, m->inv_freq.data(), m->rank, m->ranks, &m->heavy);
        if (rc) {
            m->finalized = false;
            return rc;
        }
        if (m->ranks > 1) heavy_arena(m->heavy, &m->arena, &m->arena_bytes);
        m->peer[m->rank] = m->arena;
        m->connected = m->ranks == 1;
        return mr_model_reset(m);
    }
    if (!is_engine_family(m->cfg)) {
        // resident weights only; the host drives the op kernels (tensor_ops.cu)
        m->op_path = true;
        m->finalized = true;
        return MR_OK;
    }
    const mr_model_config &c = m->cfg;
    int rc = MR_OK;
    const int H = c.query_heads, d = c.head_dim;
    MR_REQUIRE(H <= 64, "query_heads %d above the engine limit 64", H);
    MR_REQUIRE(c.hidden_size <= kRowBatch * m->grid, "hidden size %d above the engine limit %d (rows per CTA)",
               c.hidden_size, kRowBatch * m->grid);
    MR_REQUIRE(d <= 128, "head_dim %d above the engine limit 128", d);
    const int max_kvh = *std::max_element(m->layer_kvh.begin(), m->layer_kvh.end());
    const int gq_max = H / *std::min_element(m->layer_kvh.begin(), m->layer_kvh.end());
    // shared memory: control block, scratch (GEMV input vector / attention tiles), weight ring
    int max_cols = 0;
    for (auto &kv : m->tensors)
        if (kv.second.shape.size() == 2) max_cols = std::max(max_cols, (int)kv.second.shape[1]);
    // The attention region overlays the GEMV input vector: a phase's first key
    // tile is requested only after the compute barrier that ends the preceding
    // GEMV phase, and a GEMV phase reads its input only after the barrier that
    // ends the attention phase before it.  The ring gets what the overlay frees.
    m->attn_base = 0;
    m->scratch_floats = std::max((max_cols + 31) & ~31, attn_layout(gq_max, d).total);
    const size_t control = decode_control_bytes();
    const size_t scratch = ((size_t)m->scratch_floats * 4 + 127) & ~size_t(127);
    const long long ring = (long long)kSmemLimit - 1024 - (long long)control - (long long)scratch;
    MR_REQUIRE(ring >= 16 * 1024, "model too wide for the decode kernel's shared memory (input width %d)", max_cols);
    m->ring_bytes = (int)(ring & ~127ll);
    m->smem_bytes = control + scratch + (size_t)m->ring_bytes;
    auto falloc = [&](size_t n) { return static_cast<float *>(device_alloc(m, n * sizeof(float), &rc)); };
    m->d_inv_freq = falloc(d / 2);
    // The exchange buffers (and the logits) live in one arena: with tensor
    // parallelism every rank maps every other rank's arena and stores a word
    // at the same offset of each.
    {
        size_t off = 0;
        auto take = [&](size_t bytes) {
            const size_t at = off;
            off += (bytes + 255) & ~size_t(255);
            return at;
        };
        const size_t o_x = take(sizeof(Word) * c.hidden_size), o_q = take(sizeof(Word) * H * d),
                     o_k = take(sizeof(Word) * max_kvh * d), o_v = take(sizeof(Word) * max_kvh * d),
                     o_f = take(sizeof(Word) * c.ffn_dim), o_a = take(sizeof(Word) * H * d),
                     o_lat = take(sizeof(Word) * std::max(1, c.latent_dim)),
                     o_p = take(sizeof(Word) * H * kMaxAttnChunks * (d + 2)),
                     o_l = take(sizeof(float) * 64 * (size_t)c.vocab_size), o_b = take(sizeof(Word) * 4 * kMaxRanks);
        m->arena = static_cast<char *>(device_alloc(m, off, &rc));
        if (rc) return rc;
        MR_CUDA_TRY(cudaMemset(m->arena, 0, off));
        m->arena_bytes = off;
        m->x = reinterpret_cast<Word *>(m->arena + o_x);
        m->q_raw = reinterpret_cast<Word *>(m->arena + o_q);
        m->k_raw = reinterpret_cast<Word *>(m->arena + o_k);
        m->v_raw = reinterpret_cast<Word *>(m->arena + o_v);
        m->ffn = reinterpret_cast<Word *>(m->arena + o_f);
        m->latent = reinterpret_cast<Word *>(m->arena + o_lat);
        m->attn_out = reinterpret_cast<Word *>(m->arena + o_a);
        m->partial = reinterpret_cast<Word *>(m->arena + o_p);
        m->logits = reinterpret_cast<float *>(m->arena + o_l);
        m->best_slots = reinterpret_cast<Word *>(m->arena + o_b);
        m->peer[m->rank] = m->arena;
        m->connected = m->ranks == 1;
    }
    m->logits_rows = 64;
    m->state = static_cast<StepState *>(device_alloc(m, sizeof(StepState), &rc));
    if (rc) return rc;
    m->k_cache.resize(c.layers);
    m->v_cache.resize(c.layers);
    m->cache_capacity.resize(c.layers);
    for (int l = 0; l < c.layers; ++l) {
        // model.py:105: capacity = min(window or context, context); FlashLighting's
        // window applies to every layer (model.py:167)
        const int w = is_lighting(c) ? c.window : m->layer_window[l];
        const int cap = std::min(w > 0 ? w : c.context_length, c.context_length);
        m->cache_capacity[l] = cap;
        const size_t n = (size_t)m->layer_kvh[l] * cap * d;
        m->k_cache[l] = falloc(n);
        m->v_cache[l] = falloc(n);
        if (rc) return rc;
    }
    MR_CUDA_TRY(cudaMemcpy(m->d_inv_freq, m->inv_freq.data(), sizeof(float) * (d / 2), cudaMemcpyHostToDevice));
    // Attention unit u runs on CTA u.  Those CTAs own no rows of the q/k/v,
    // o and down phases (nor residual rows), so that they go from one
    // attention phase's neighbours to the next without a GEMV of their own:
    // the fewest units any layer has at full context, unless that is more
    // than a quarter of the grid.
    int skip = m->grid;
    for (int l = 0; l < c.layers; ++l) {
        // this rank's KV heads of the layer (none when the layer has fewer heads than ranks)
        int kv_lo, kv_n;
        rank_rows(m->layer_kvh[l], m->rank, m->ranks, kv_lo, kv_n);
        skip = kv_n > 0 ? std::min(skip, kv_n * attn_chunks(m->cache_capacity[l], kv_n, m->grid)) : 0;
    }
    if (skip > m->grid / 4) skip = 0;  // too many units to spare their CTAs: no CTA is set aside
    m->xres_skip = skip;
    rank_rows(c.hidden_size, m->rank, m->ranks, m->xres_lo, m->xres_n);
    MR_REQUIRE((m->xres_n + m->grid - skip - 1) / (m->grid - skip) <= kRowBatch,
               "hidden size %d above the engine limit (rows per CTA)", c.hidden_size);
    rc = setup_aux(m);
    if (!rc) rc = build_plan(m);
    if (!rc) rc = build_pieces(m);
    if (!rc) rc = build_groups(m);
    if (rc) return rc;
    m->d_phases = static_cast<Phase *>(device_alloc(m, sizeof(Phase) * m->phases.size(), &rc));
    if (rc) return rc;
    MR_CUDA_TRY(cudaMemcpy(m->d_phases, m->phases.data(), sizeof(Phase) * m->phases.size(), cudaMemcpyHostToDevice));
    MR_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void *>(decode_step_kernel),
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->smem_bytes));
    int per_sm = 0;
    MR_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void *>(decode_step_kernel),
                                                              kBlockThreads, m->smem_bytes));
    MR_REQUIRE(per_sm >= 1, "decode kernel cannot be resident (occupancy 0)");
    MR_CUDA_TRY(cudaEventCreate(&m->ev0));
    MR_CUDA_TRY(cudaEventCreate(&m->ev1));
    MR_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&m->h_ids), sizeof(int) * (mr_model::kHostIds + 32),
                              cudaHostAllocDefault));
    m->h_error = m->h_ids + mr_model::kHostIds;
    MR_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&m->h_logits), sizeof(float) * c.vocab_size,
                              cudaHostAllocDefault));
    setup_prefill(m);
    m->finalized = true;
    return mr_model_reset(m);
}

int mr_model_set_tensor_parallel(mr_model *m, int rank, int ranks) {
    MR_REQUIRE(m, "model is NULL");
    MR_REQUIRE(!m->finalized, "tensor parallelism is set before mr_model_finalize");
    MR_REQUIRE(ranks >= 1 && ranks <= kMaxRanks && rank >= 0 && rank < ranks, "rank %d of %d ranks (at most %d)",
               rank, ranks, kMaxRanks);
    MR_REQUIRE(ranks == 1 || is_engine_family(m->cfg) || m->cfg.family == MR_FAMILY_HEAVY_MEDIUM_20,
               "tensor / expert parallelism needs a decode-engine family or heavy-medium-2.0");
    m->rank = rank;
    m->ranks = ranks;
    return MR_OK;
}

int mr_model_tp_handle(mr_model *m, void *handle, size_t bytes) {
    MR_REQUIRE(m && handle, "NULL argument");
    MR_REQUIRE(m->finalized && m->arena, "model is not finalized");
    MR_REQUIRE(bytes >= sizeof(cudaIpcMemHandle_t), "handle buffer needs %zu bytes", sizeof(cudaIpcMemHandle_t));
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    cudaIpcMemHandle_t h;
    MR_CUDA_TRY(cudaIpcGetMemHandle(&h, m->arena));
    memcpy(handle, &h, sizeof(h));
    return MR_OK;
}

int mr_model_tp_connect(mr_model *m, const void *handles, size_t bytes_each) {
    MR_REQUIRE(m && handles, "NULL argument");
    MR_REQUIRE(m->finalized && m->arena, "model is not finalized");
    MR_REQUIRE(bytes_each >= sizeof(cudaIpcMemHandle_t), "handles of %zu bytes, need %zu", bytes_each,
               sizeof(cudaIpcMemHandle_t));
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    for (int j = 0; j < m->ranks; ++j) {
        if (j == m->rank || m->peer_open[j]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + (size_t)j * bytes_each, sizeof(h));
        void *p = nullptr;
        MR_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        m->peer[j] = static_cast<char *>(p);
        m->peer_open[j] = true;
    }
    if (m->heavy) heavy_connect(m->heavy, m->peer);
    m->connected = true;
    return MR_OK;
}

int mr_model_set_batched_prefill(mr_model *m, int enable, int *available) {
    MR_REQUIRE(m, "model is NULL");
    MR_REQUIRE(enable >= 0 && enable <= 2, "enable must be 0, 1 or 2");
    m->prefill_on = enable != 0;
    m->pw.tcgen05 = enable != 2;
    if (available) *available = (m->heavy ? heavy_batchable(m->heavy) : m->prefill_ok) ? 1 : 0;
    return MR_OK;
}

int mr_model_reset(mr_model *m) {
    MR_REQUIRE(m, "model is NULL");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    if (!m->finalized) return set_error(MR_ERR_STATE, "model is not finalized");
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    if (!m->op_path && !m->heavy) {
        MR_CUDA_TRY(cudaMemset(m->state, 0, sizeof(StepState)));
        MR_CUDA_TRY(cudaMemcpy(&m->state->wait_limit_ns, &m->wait_limit_ns, sizeof(m->wait_limit_ns),
                               cudaMemcpyHostToDevice));
    }
    if (m->heavy) {
        const int rc = heavy_reset(m->heavy);
        if (rc) return rc;
    }
    if (const int rc = reset_aux(m)) return rc;
    m->position = 0;
    m->failed = false;
    return MR_OK;
}

int mr_model_position(const mr_model *m, int *position) {
    MR_REQUIRE(m && position, "NULL argument");
    *position = m->position;
    return MR_OK;
}

int mr_model_weight_bytes(const mr_model *m, uint64_t *bytes) {
    MR_REQUIRE(m && bytes, "NULL argument");
    uint64_t total = 0;
    for (auto &kv : m->tensors) total += kv.second.bytes;
    *bytes = total;
    return MR_OK;
}

int mr_model_step(mr_model *m, int token, float *logits_out, int *argmax_out) {
    int rc = ready(m);
    if (rc) return rc;
    if (m->heavy) {
        std::vector<float> row(m->cfg.vocab_size);
        rc = heavy_feed(m, &token, 1, 0, row.data());
        if (rc) return rc;
        if (logits_out) memcpy(logits_out, row.data(), sizeof(float) * row.size());
        if (argmax_out) *argmax_out = host_argmax(row.data(), (int)row.size());
        return MR_OK;
    }
    rc = run_feed(m, &token, 1, 0, logits_out);
    if (rc) return rc;
    if (argmax_out) {
        StepState s;
        MR_CUDA_TRY(cudaMemcpy(&s, m->state, sizeof(s), cudaMemcpyDeviceToHost));
        *argmax_out = s.last_argmax;
    }
    return MR_OK;
}

int mr_model_prefill(mr_model *m, const int *ids, int n, int return_all, float *out) {
    int rc = ready(m);
    if (rc) return rc;
    MR_REQUIRE(ids && n > 0, "input_ids must be a non-empty 1D integer sequence");
    if (m->heavy) return heavy_feed(m, ids, n, return_all, out);
    return run_feed(m, ids, n, return_all, out);
}

int mr_model_generate_greedy(mr_model *m, const int *ids, int n, int max_new, int eos, int *out_tokens,
                             int *out_count, int *out_nonfinite) {
    int rc = ready(m);
    if (rc) return rc;
    MR_REQUIRE(ids && n > 0 && out_tokens && out_count && out_nonfinite, "NULL argument");
    MR_REQUIRE(max_new > 0, "max_new must be positive");
    const int V = m->cfg.vocab_size;
    for (int i = 0; i < n; ++i) MR_REQUIRE(ids[i] >= 0 && ids[i] < V, "input token is outside the vocabulary");
    MR_REQUIRE(m->position + n + max_new - 1 <= m->cfg.context_length,
               "prompt plus requested generation exceeds context_length");
    if (m->heavy) {  // greedy on the host over the device token step (model.py:318-357)
        std::vector<float> row(V);
        *out_count = 0;
        *out_nonfinite = 0;
        rc = heavy_feed(m, ids, n, 0, row.data());
        for (int i = 0; !rc && i < max_new; ++i) {
            for (float v : row)
                if (!std::isfinite(v)) {
                    *out_nonfinite = 1;
                    return MR_OK;
                }
            const int token = host_argmax(row.data(), V);
            out_tokens[(*out_count)++] = token;
            if (token == eos || i + 1 == max_new) break;
            rc = heavy_feed(m, &token, 1, 0, row.data());
        }
        return rc;
    }
    rc = ensure_feed(m, n);
    if (!rc) rc = ensure_gen(m, max_new);
    if (rc) return rc;
    MR_CUDA_TRY(cudaMemcpyAsync(m->feed, ids, sizeof(int) * n, cudaMemcpyHostToDevice, m->ctx->stream));
    StepControl ctl = base_control(m);
    ctl.feed_len = n;
    ctl.gen_max = max_new;
    ctl.eos = eos;
    ctl.gen_out = m->gen_out;
    for (int i = 0; i < n + max_new - 1; ++i) {
        rc = launch_step(m, ctl);
        if (rc) {
            m->failed = true;
            return rc;
        }
    }
    rc = sync_and_check(m, "generate");
    if (rc) return rc;
    StepState s;
    MR_CUDA_TRY(cudaMemcpy(&s, m->state, sizeof(s), cudaMemcpyDeviceToHost));
    *out_count = s.gen_count;
    *out_nonfinite = s.nonfinite;
    if (s.gen_count) MR_CUDA_TRY(cudaMemcpy(out_tokens, m->gen_out, sizeof(int) * s.gen_count, cudaMemcpyDeviceToHost));
    m->position = s.position;
    // leave the state ready for further decode calls
    MR_CUDA_TRY(cudaMemset(&m->state->stopped, 0, sizeof(int)));
    MR_CUDA_TRY(cudaMemset(&m->state->gen_count, 0, sizeof(int)));
    return MR_OK;
}

int mr_model_generate_sampled(mr_model *m, const int *ids, int n, int max_new, int eos, double temperature,
                              int top_k, double top_p, const uint64_t *pcg_state, int *out_tokens, int *out_count,
                              int *out_nonfinite) {
    int rc = ready(m);
    if (rc) return rc;
    MR_REQUIRE(ids && n > 0 && pcg_state && out_tokens && out_count && out_nonfinite, "NULL argument");
    MR_REQUIRE(max_new > 0, "max_new must be positive");
    MR_REQUIRE(std::isfinite(temperature) && temperature >= 0, "temperature must be finite and non-negative");
    MR_REQUIRE(top_k >= 0 && std::isfinite(top_p) && top_p > 0 && top_p <= 1,
               "top_k must be non-negative and top_p must be in (0,1]");
    MR_REQUIRE(m->ranks == 1, "device sampling runs on one GPU");
    const int V = m->cfg.vocab_size;
    for (int i = 0; i < n; ++i) MR_REQUIRE(ids[i] >= 0 && ids[i] < V, "input token is outside the vocabulary");
    MR_REQUIRE(eos >= 0 && eos < V, "eos_token_id is outside vocabulary");
    MR_REQUIRE(m->position + n + max_new - 1 <= m->cfg.context_length,
               "prompt plus requested generation exceeds context_length");
    if (!m->sampler && (rc = sampler_create(V, &m->sampler))) return rc;
    if ((rc = ensure_gen(m, max_new))) return rc;
    cudaStream_t st = m->ctx->stream;
    const unsigned long long pcg[4] = {pcg_state[0], pcg_state[1], pcg_state[2], pcg_state[3]};
    if ((rc = sampler_seed(m->sampler, st, pcg))) return rc;
    const SampleParams sp{temperature, top_p, top_k, eos, max_new};
    *out_count = 0;
    *out_nonfinite = 0;
    int count = 0, nonfinite = 0;
    if (m->heavy) {
        // prompt (batched where it applies), then per token: sample on the device, the
        // step from the sampled id; the host reads back only the stop state
        const bool batched = n > 1 && m->prefill_on && heavy_batchable(m->heavy);
        rc = heavy_feed(m, ids, n, 0, nullptr);
        const float *logits = batched ? heavy_prefill_logits(m->heavy) : heavy_logits(m->heavy);
        for (int i = 0; !rc && i < max_new; ++i) {
            rc = sampler_step(m->sampler, st, logits, sp, heavy_token_slot(m->heavy), m->gen_out, nullptr);
            if (!rc) rc = sampler_result(m->sampler, st, &count, &nonfinite);
            if (rc || nonfinite || count < i + 1 || count == max_new || i + 1 == max_new) break;
            int token = 0;
            MR_CUDA_TRY(cudaMemcpy(&token, m->gen_out + i, sizeof(int), cudaMemcpyDeviceToHost));
            if (token == eos) break;
            rc = heavy_token_from_slot(m->heavy, m->position);
            if (!rc) {
                ++m->position;
                logits = heavy_logits(m->heavy);
            }
        }
        if (!rc) {
            const cudaError_t err = cudaStreamSynchronize(st);
            rc = err != cudaSuccess ? cuda_error(err, "heavy-medium-2.0 sampling") : heavy_status(m->heavy);
        }
        if (rc) {
            m->failed = true;
            return rc;
        }
    } else {
        // prompt, then sample -> step -> sample ... queued without a synchronise: the step
        // reads its token from the step state the sampler writes, and skips once stopped
        const bool batched = m->prefill_ok && m->prefill_on && n > 1;
        if ((rc = run_feed(m, ids, n, 0, nullptr))) return rc;
        const float *logits = batched ? m->pw.logits : m->logits;
        StepControl ctl = base_control(m);
        for (int i = 0; i < max_new; ++i) {
            rc = sampler_step(m->sampler, st, logits, sp, &m->state->token, m->gen_out, &m->state->stopped);
            if (!rc && i + 1 < max_new) rc = launch_step(m, ctl);
            if (rc) {
                m->failed = true;
                return rc;
            }
            logits = m->logits;
        }
        if ((rc = sync_and_check(m, "generate"))) return rc;
        if ((rc = sampler_result(m->sampler, st, &count, &nonfinite))) return rc;
        StepState s;
        MR_CUDA_TRY(cudaMemcpy(&s, m->state, sizeof(s), cudaMemcpyDeviceToHost));
        m->position = s.position;
        MR_CUDA_TRY(cudaMemset(&m->state->stopped, 0, sizeof(int)));  // ready for further decode calls
    }
    *out_count = count;
    *out_nonfinite = nonfinite;
    if (count) MR_CUDA_TRY(cudaMemcpy(out_tokens, m->gen_out, sizeof(int) * count, cudaMemcpyDeviceToHost));
    return MR_OK;
}

int mr_model_layer_state(const mr_model *m, int layer, int loop, mr_layer_state *out) {
    MR_REQUIRE(m && out, "NULL argument");
    MR_REQUIRE(layer >= 0 && layer < m->cfg.layers, "layer out of range");
    MR_REQUIRE(loop >= 0 && loop < std::max(1, m->cfg.inner_loop_steps), "loop out of range");
    memset(out, 0, sizeof(*out));
    out->present = m->position > 0;
    if (!out->present || !m->finalized) return MR_OK;
    const int cap = m->heavy ? m->cfg.context_length : m->cache_capacity[layer];
    out->ring_count = m->position;
    out->ring_capacity = cap;
    out->ring_length = std::min(m->position, cap);
    out->ring_start = (m->position - out->ring_length) % cap;
    if (is_lighting_ring(m->cfg)) {  // the latent cache after this step's compaction (drop path)
        out->latent_rows = out->ring_length;
        out->memory_size = 0;
    }
    if (m->aux_on) {  // relay rows (flashnano-1.6) or memory rows (FlashLighting), read back
        int count = 0;
        MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
        MR_CUDA_TRY(cudaMemcpy(&count, m->aux_host[layer].relay_count, sizeof(int), cudaMemcpyDeviceToHost));
        if (is_cbr(m->cfg)) {
            out->relay_count = count;
        } else {
            out->memory_size = count;
            out->latent_rows = count + out->ring_length;
        }
    }
    return MR_OK;
}

}  // extern "C"

namespace {
// FlashLighting with memory slots: positions and token counts of the memory rows
// (logical order), then the window's rows (one token each).
int latent_rows(const mr_model *m, int layer, std::vector<int> &pos, std::vector<float> &cnt) {
    pos.clear();
    cnt.clear();
    const int n = std::min(m->position, m->cache_capacity[layer]);
    if (m->aux_on) {
        const aux::Layer &L = m->aux_host[layer];
        int size = 0;
        MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
        MR_CUDA_TRY(cudaMemcpy(&size, L.relay_count, sizeof(int), cudaMemcpyDeviceToHost));
        pos.resize(size);
        cnt.resize(size);
        if (size) {
            MR_CUDA_TRY(cudaMemcpy(pos.data(), L.mem_pos, sizeof(int) * size, cudaMemcpyDeviceToHost));
            MR_CUDA_TRY(cudaMemcpy(cnt.data(), L.mem_cnt, sizeof(float) * size, cudaMemcpyDeviceToHost));
        }
    }
    for (int i = 0; i < n; ++i) {
        pos.push_back(m->position - n + i);
        cnt.push_back(1.0f);
    }
    return MR_OK;
}
}  // namespace

extern "C" {

int mr_model_latent_positions(const mr_model *m, int layer, int *out, int capacity, int *rows) {
    MR_REQUIRE(m && rows, "NULL argument");
    MR_REQUIRE(layer >= 0 && layer < m->cfg.layers, "layer out of range");
    *rows = 0;
    if (!m->finalized || m->op_path || !is_lighting(m->cfg))
        return set_error(MR_ERR_ARGUMENT, "model has no latent cache");
    std::vector<int> pos;
    std::vector<float> cnt;
    if (int rc = latent_rows(m, layer, pos, cnt)) return rc;
    const int n = static_cast<int>(pos.size());
    MR_REQUIRE(out || n == 0, "NULL argument");
    MR_REQUIRE(capacity >= n, "positions buffer holds %d rows, need %d", capacity, n);
    for (int i = 0; i < n; ++i) out[i] = pos[i];
    *rows = n;
    return MR_OK;
}

int mr_model_latent_counts(const mr_model *m, int layer, float *out, int capacity, int *rows) {
    MR_REQUIRE(m && rows, "NULL argument");
    MR_REQUIRE(layer >= 0 && layer < m->cfg.layers, "layer out of range");
    *rows = 0;
    if (!m->finalized || m->op_path || !is_lighting(m->cfg))
        return set_error(MR_ERR_ARGUMENT, "model has no latent cache");
    std::vector<int> pos;
    std::vector<float> cnt;
    if (int rc = latent_rows(m, layer, pos, cnt)) return rc;
    const int n = static_cast<int>(cnt.size());
    MR_REQUIRE(out || n == 0, "NULL argument");
    MR_REQUIRE(capacity >= n, "counts buffer holds %d rows, need %d", capacity, n);
    for (int i = 0; i < n; ++i) out[i] = cnt[i];
    *rows = n;
    return MR_OK;
}

int mr_model_last_topk(const mr_model *m, int layer, int loop, int *blocks, int capacity) {
    MR_REQUIRE(m && blocks, "NULL argument");
    if (!m->heavy) return set_error(MR_ERR_ARGUMENT, "model has no sparse block attention");
    MR_REQUIRE(layer >= 0 && layer < m->cfg.layers && loop >= 0 && loop < std::max(1, m->cfg.inner_loop_steps),
               "layer / loop out of range");
    return heavy_last_topk(m->heavy, layer, loop, blocks, capacity);
}

int mr_model_last_experts(const mr_model *m, int layer, int loop, int *experts, float *weights, int capacity) {
    MR_REQUIRE(m && experts && weights, "NULL argument");
    if (!m->heavy) return set_error(MR_ERR_ARGUMENT, "model has no experts");
    MR_REQUIRE(layer >= 0 && layer < m->cfg.layers && loop >= 0 && loop < std::max(1, m->cfg.inner_loop_steps),
               "layer / loop out of range");
    return heavy_last_experts(m->heavy, layer, loop, experts, weights, capacity);
}

int mr_model_set_log1p_table(mr_model *m, const float *values, int n) {
    MR_REQUIRE(m && values, "NULL argument");
    if (!m->heavy) return set_error(MR_ERR_ARGUMENT, "model has no sparse block attention");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    return heavy_set_log1p(m->heavy, values, n);
}

int mr_model_set_wait_limit(mr_model *m, uint64_t nanoseconds) {
    MR_REQUIRE(m, "model is NULL");
    MR_REQUIRE(m->finalized, "model is not finalized");
    MR_REQUIRE(nanoseconds >= 1000000ull, "a device wait limit below 1 ms would fail ordinary steps");
    MR_CUDA_TRY(cudaSetDevice(m->ctx->device));
    MR_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    m->wait_limit_ns = nanoseconds;
    if (m->heavy) return heavy_set_wait_limit(m->heavy, nanoseconds);
    if (!m->op_path)
        MR_CUDA_TRY(cudaMemcpy(&m->state->wait_limit_ns, &m->wait_limit_ns, sizeof(m->wait_limit_ns),
                               cudaMemcpyHostToDevice));
    return MR_OK;
}

int mr_model_inject_fault(mr_model *m, int phase) {
    MR_REQUIRE(m, "model is NULL");
    MR_REQUIRE(m->finalized, "model is not finalized");
    MR_REQUIRE(!m->op_path, "the host-stepped families have no device waits to exercise");
    MR_REQUIRE(phase >= -1, "phase must be -1 (off) or a phase index");
    if (m->heavy) return heavy_inject_fault(m->heavy, phase >= 0);
    MR_REQUIRE(phase < static_cast<int>(m->phases.size()) - 1, "phase %d outside the step's %d phases", phase,
               static_cast<int>(m->phases.size()) - 1);
    m->withhold_phase = phase;
    return MR_OK;
}

int mr_model_trace_decode(mr_model *m, int token, uint64_t *stamps, int capacity, int *phases, int *grid) {
    int rc = ready(m);
    if (rc) return rc;
    MR_REQUIRE(stamps && phases && grid, "NULL argument");
    MR_REQUIRE(token >= 0 && token < m->cfg.vocab_size, "token outside the vocabulary");
    MR_REQUIRE(m->position + 1 <= m->cfg.context_length, "context_length exceeded");
    if (m->heavy) {  // kernel-boundary stamps of the device token step
        int count = 0;
        rc = heavy_trace_token(m->heavy, token, m->position, reinterpret_cast<unsigned long long *>(stamps),
                               capacity, &count);
        if (rc) {
            m->failed = true;
            return rc;
        }
        m->position += 1;
        *phases = count - 1;
        *grid = 0;
        return MR_OK;
    }
    const int executed = (int)m->phases.size() - 1;  // every phase but the step end
    const size_t need = 1 + (size_t)executed * ((size_t)m->grid * kTraceStamps + 1);
    MR_REQUIRE((size_t)capacity >= need, "trace needs %zu stamps", need);
    rc = ensure_feed(m, 1);
    if (rc) return rc;
    unsigned long long *d_trace = nullptr;
    MR_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void **>(&d_trace), need * sizeof(unsigned long long),
                                m->ctx->stream));
    MR_CUDA_TRY(cudaMemcpyAsync(m->feed, &token, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
    StepControl ctl = base_control(m);
    ctl.feed_len = 1;
    ctl.trace = d_trace;
    rc = launch_step(m, ctl);
    if (!rc) rc = sync_and_check(m, "trace");
    if (!rc) {
        cudaError_t err = cudaMemcpy(stamps, d_trace, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        if (err != cudaSuccess) rc = cuda_error(err, "trace copy");
    }
    cudaFreeAsync(d_trace, m->ctx->stream);
    if (rc) return rc;
    m->position += 1;
    *phases = executed;
    *grid = m->grid;
    return MR_OK;
}

int mr_model_bench_decode(mr_model *m, int first_token, int steps, float *device_ms) {
    int rc = ready(m);
    if (rc) return rc;
    MR_REQUIRE(device_ms && steps > 0, "bad arguments");
    MR_REQUIRE(first_token >= 0 && first_token < m->cfg.vocab_size, "token outside the vocabulary");
    MR_REQUIRE(m->position + steps <= m->cfg.context_length, "decode steps exceed context_length");
    if (m->heavy) {
        if (!m->ev0) MR_CUDA_TRY(cudaEventCreate(&m->ev0));
        if (!m->ev1) MR_CUDA_TRY(cudaEventCreate(&m->ev1));
        MR_CUDA_TRY(cudaEventRecord(m->ev0, m->ctx->stream));
        rc = heavy_greedy_chain(m->heavy, first_token, m->position, steps);
        if (!rc) MR_CUDA_TRY(cudaEventRecord(m->ev1, m->ctx->stream));
        const cudaError_t err = cudaStreamSynchronize(m->ctx->stream);
        if (!rc && err == cudaSuccess) rc = heavy_status(m->heavy);
        if (rc || err != cudaSuccess) {
            m->failed = true;
            return rc ? rc : cuda_error(err, "heavy-medium-2.0 decode");
        }
        MR_CUDA_TRY(cudaEventElapsedTime(device_ms, m->ev0, m->ev1));
        m->position += steps;
        return MR_OK;
    }
    rc = ensure_feed(m, 1);
    if (!rc) rc = ensure_gen(m, steps);
    if (rc) return rc;
    MR_CUDA_TRY(cudaMemcpyAsync(m->feed, &first_token, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
    StepControl ctl = base_control(m);
    ctl.feed_len = 1;
    ctl.gen_max = steps + 1;
    ctl.gen_out = m->gen_out;
    MR_CUDA_TRY(cudaEventRecord(m->ev0, m->ctx->stream));
    for (int i = 0; i < steps; ++i) {
        rc = launch_step(m, ctl);
        if (rc) {
            m->failed = true;
            return rc;
        }
    }
    MR_CUDA_TRY(cudaEventRecord(m->ev1, m->ctx->stream));
    rc = sync_and_check(m, "bench");
    if (rc) return rc;
    MR_CUDA_TRY(cudaEventElapsedTime(device_ms, m->ev0, m->ev1));
    StepState s;
    MR_CUDA_TRY(cudaMemcpy(&s, m->state, sizeof(s), cudaMemcpyDeviceToHost));
    m->position = s.position;
    MR_CUDA_TRY(cudaMemset(&m->state->stopped, 0, sizeof(int)));
    MR_CUDA_TRY(cudaMemset(&m->state->gen_count, 0, sizeof(int)));
    return MR_OK;
}

}  // extern "C"
