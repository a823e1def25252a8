"""Float64 restatement of the token loop for the full-size parity fixtures.

TEST INFRASTRUCTURE ONLY (the checker, never the thing measured).

At the BASELINE architectures' depth and width the reference's own float32
logits are up to 5e-5 away from the exact values (FlashLighting: 0.15% of
them further than the parity tolerance of the exact value), so a float32
implementation that sums in any other order cannot stay within atol 2e-5 of
the reference everywhere, however accurate it is.  This script computes the
exact values (float64 arithmetic over the same synthetic weights, prompt and
greedy tokens) so that the GPU tests can check the device against them at the
north-star tolerance, and against the reference at that tolerance plus the
reference's own measured deviation.

It restates the reference's algorithm (miracle_reasoning/model.py) family by
family in NumPy float64:

* grouped-query families (_gqa, model.py:95-116; _step, 257-285): RMSNorm,
  q/k norm per head, RoPE (interleaved or split-half, config.py's inverse
  frequencies), the local ring or the full cache, softmax attention, SwiGLU;
* FlashLighting (_lighting, model.py:146-190) on the drop path (memory_slots
  0; the fixtures stay inside the window, so no latent is dropped);
* Heavy Medium (_heavy_attention and _moe, model.py:192-255): the kept blocks
  and the chosen experts (count and ids) are the reference's own, read from
  bench_heavy.npz, so the float64 values follow the reference's discrete
  path; the expert weights are recomputed in float64 from the router.

    python tests/golden/make_exact.py [--only lite lighting nano17_window heavy]

Writes tests/golden/exact_<case>.npz: per stored step the float64 logits at
the bench fixture's positions (leading 1024, every 16th, the reference's
top-64 ids).
"""
from __future__ import annotations

import argparse
import json
import math
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def rms(x, gain, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * (1.0 if gain is None else gain)


def rope(x, position, freq, heads, d, split_half):
    x = x.reshape(heads, d).copy()
    angle = position * np.asarray(freq, np.float64)
    c, s = np.cos(angle), np.sin(angle)
    if split_half:
        u, v = x[:, :d // 2].copy(), x[:, d // 2:].copy()
        x[:, :d // 2], x[:, d // 2:] = u * c - v * s, u * s + v * c
    else:
        u, v = x[:, 0::2].copy(), x[:, 1::2].copy()
        x[:, 0::2], x[:, 1::2] = u * c - v * s, u * s + v * c
    return x.reshape(-1)


def softmax_mix(scores, values):
    p = np.exp(scores - scores.max())
    return (p / p.sum()) @ values


class F64Weights:
    """Tensors of the synthetic model in float64, generated on first use (a
    bounded cache: the Heavy Medium model is 73 GB in BF16)."""

    def __init__(self, config, stored, budget_bytes=24 << 30):
        from collections import OrderedDict
        self.config, self.stored = config, stored
        self.plan = {n: (i, s, std) for i, n, s, std in cases.synthetic.tensor_plan(config)}
        self.cache, self.used, self.budget = OrderedDict(), 0, budget_bytes
        self.f32 = cases.synthetic.synthetic_weights(config, "F32") if stored == "F32" else None

    def __getitem__(self, name):
        if name in self.cache:
            self.cache.move_to_end(name)
            return self.cache[name]
        index, shape, std = self.plan[name]
        if std is None:
            value = np.ones(shape, np.float64)
        elif self.f32 is not None:
            value = np.asarray(self.f32[name], np.float64)
        else:
            bits = cases.synthetic.hash_normal_bf16(0, index, shape, std)
            value = cases.widen_bf16(bits).astype(np.float64)
        while self.cache and self.used + value.nbytes > self.budget:
            _, old = self.cache.popitem(last=False)
            self.used -= old.nbytes
        self.cache[name] = value
        self.used += value.nbytes
        return value


def gqa_layer(c, W, p, layer, h, i, state, ctx, freq):
    kvh, d = c.layer_kv_heads(layer), c.head_dim
    a = rms(h, W[p + "a_norm"], c.norm_eps)
    q, k, v = W[p + "q"] @ a, W[p + "k"] @ a, W[p + "v"] @ a
    if c.qk_norm:
        q = np.concatenate([rms(x, W[p + "q_norm"], c.norm_eps) for x in q.reshape(-1, d)])
        k = np.concatenate([rms(x, W[p + "k_norm"], c.norm_eps) for x in k.reshape(-1, d)])
    split = c.split_half_rope
    q, k = rope(q, i, freq, c.query_heads, d, split), rope(k, i, freq, kvh, d, split)
    state.setdefault("keys", []).append(k)
    state.setdefault("values", []).append(v)
    cap = min(c.layer_window(layer) or ctx, ctx)
    keys = np.stack(state["keys"][-cap:]).reshape(-1, kvh, d)
    vals = np.stack(state["values"][-cap:]).reshape(-1, kvh, d)
    group = c.query_heads // kvh
    att = np.concatenate([softmax_mix(keys[:, hh // group] @ q[hh * d:(hh + 1) * d] / math.sqrt(d), vals[:, hh // group])
                          for hh in range(c.query_heads)])
    h = h + c.residual_scale * (W[p + "o"] @ att)
    f = rms(h, W[p + "f_norm"], c.norm_eps)
    g, u = W[p + "ffn.gate"] @ f, W[p + "ffn.up"] @ f
    return h + c.residual_scale * (W[p + "ffn.down"] @ (g / (1 + np.exp(-g)) * u))


def lighting_layer(c, W, p, layer, h, i, state, ctx, freq):
    d, H, KV = c.head_dim, c.query_heads, c.kv_heads
    a = rms(h, W[p + "a_norm"], c.norm_eps)
    q = np.concatenate([rms(x, W[p + "q_norm"], c.norm_eps) for x in (W[p + "q"] @ a).reshape(-1, d)])
    q = rope(q, i, freq, H, d, True)
    latent = rms(W[p + "latent"] @ a, W[p + "latent_norm"], c.norm_eps)
    state.setdefault("latents", []).append(latent)
    state.setdefault("positions", []).append(i)
    if c.memory_slots != 0 or len(state["latents"]) > c.window:
        raise NotImplementedError("only the drop path inside the window is restated")
    L = np.stack(state["latents"])
    keys = np.stack([rope(np.concatenate([rms(x, W[p + "k_norm"], c.norm_eps) for x in (W[p + "k"] @ lt).reshape(-1, d)]),
                          pos, freq, KV, d, True) for lt, pos in zip(L, state["positions"])]).reshape(len(L), KV, d)
    vals = (L @ W[p + "v"].T).reshape(len(L), KV, d)
    group = H // KV
    att = np.concatenate([softmax_mix(keys[:, hh // group] @ q[hh * d:(hh + 1) * d] / math.sqrt(d), vals[:, hh // group])
                          for hh in range(H)])
    attended = W[p + "o"] @ att
    g, u = W[p + "ffn.gate"] @ a, W[p + "ffn.up"] @ a
    ffn = W[p + "ffn.down"] @ (g / (1 + np.exp(-g)) * u)
    return h + c.residual_scale * (W[p + "attention_gate"][0] * attended + W[p + "ffn_gate"][0] * ffn)


def heavy_layer(c, W, p, layer, h, i, state, ctx, freq, decisions):
    """Both inner loops of one layer; decisions[k] = the reference's (kept blocks
    per head, experts) of inner step k of this layer."""
    s, d, H, KV = c.source, c.head_dim, c.query_heads, c.kv_heads
    long = s["long_context"]
    block, width = long["global_block_size"], KV * d
    scale = c.residual_scale / math.sqrt(c.inner_loop_steps)
    loops = state.setdefault("loops", [{} for _ in range(c.inner_loop_steps)])
    for k, inner in enumerate(loops):
        kept, experts = decisions[k]
        a = rms(h, W[p + "a_norm"], c.norm_eps)
        q = np.concatenate([rms(x, None, 1e-6) for x in (W[p + "q"] @ a).reshape(-1, d)])
        kv = W[p + "kv_up"] @ (W[p + "latent"] @ a)
        key = rope(np.concatenate([rms(x, None, 1e-6) for x in kv[:width].reshape(-1, d)]), i, freq, KV, d,
                   c.split_half_rope)
        q = rope(q, i, freq, H, d, c.split_half_rope)
        inner.setdefault("k", []).append(key)
        inner.setdefault("v", []).append(kv[width:])
        count = len(inner["k"])
        length = min(c.window, count)
        K, V = np.stack(inner["k"]).reshape(count, KV, d), np.stack(inner["v"]).reshape(count, KV, d)
        blocks = (count + block - 1) // block
        mk = np.stack([K[b * block:(b + 1) * block].mean(0) for b in range(blocks)])
        mv = np.stack([V[b * block:(b + 1) * block].mean(0) for b in range(blocks)])
        end = np.minimum((np.arange(blocks) + 1) * block - 1, i)
        penalty = long.get("alibi_slope_scale", 0.015) / math.sqrt(d) * np.log1p(i - end)
        group = H // KV
        att = []
        for hh in range(H):
            kh = hh // group
            qh = q[hh * d:(hh + 1) * d]
            sw = K[count - length:, kh] @ qh / math.sqrt(d)
            sb = mk[:, kh] @ qh / math.sqrt(d) - penalty
            keep = np.asarray(kept[hh], dtype=np.int64)
            scores = np.concatenate([sw, sb[keep]])
            values = np.concatenate([V[count - length:, kh], mv[keep, kh]])
            att.append(softmax_mix(scores, values))
        h = h + scale * (W[p + "o"] @ np.concatenate(att))
        f = rms(h, W[p + "f_norm"], c.norm_eps)
        coarse = W[p + "router.coarse.weight"] @ f + W[p + "router.coarse.bias"] + W[p + "router.group_bias"]
        fine = W[p + "router.fine.weight"] @ f + W[p + "router.fine.bias"] + W[p + "router.expert_bias"]
        per_group = (s["routed_experts"] + s["router_groups"] - 1) // s["router_groups"]
        groups = np.minimum(np.arange(s["routed_experts"]) // per_group, s["router_groups"] - 1)
        logits = (fine + coarse[groups]) / max(s.get("router_temperature", 1.0), 1e-4)
        probs = np.exp(logits - logits.max())
        probs /= probs.sum()
        chosen = probs[experts]
        chosen = chosen / chosen.sum()
        result = np.zeros_like(h)

        def ffn(root):
            g, u = W[root + "gate"] @ f, W[root + "up"] @ f
            return W[root + "down"] @ (g / (1 + np.exp(-g)) * u)

        for e, w in zip(experts, chosen):
            result += w * ffn(p + f"experts.{e}.")
        for e in range(s["shared_experts"]):
            result += c.residual_scale / max(s["shared_experts"], 1) * ffn(p + f"shared.{e}.")
        h = h + scale * result
    return h


def run(name):
    config, stored, ctx, prompt, steps = cases.bench_case(name)
    golden = np.load(cases.GOLDEN_DIR / f"bench_{name}.npz")
    c = config
    W = F64Weights(c, stored)
    freq = c.inverse_frequencies()
    heavy = c.family == "heavy-medium-2.0"
    decisions = json.loads(str(golden["meta"]))["decisions"] if heavy else None
    states = [{} for _ in range(c.layers)]
    tokens = list(prompt) + [int(t) for t in golden["tokens"]]
    rows = []
    t0 = time.time()
    for i, token in enumerate(tokens):
        h = W["embed"][token].copy()
        for layer in range(c.layers):
            p = f"layers.{layer}."
            if heavy:
                steps_of = [(decisions[i]["topk"][layer * c.inner_loop_steps + k],
                             decisions[i]["experts"][layer * c.inner_loop_steps + k]) for k in range(c.inner_loop_steps)]
                h = heavy_layer(c, W, p, layer, h, i, states[layer], ctx, freq, steps_of)
            elif c.family == "flashlighting-2.0":
                h = lighting_layer(c, W, p, layer, h, i, states[layer], ctx, freq)
            else:
                h = gqa_layer(c, W, p, layer, h, i, states[layer], ctx, freq)
        if i >= len(prompt) - 1:
            head = W["embed"] if c.tie_embeddings else W["output"]
            rows.append(head @ rms(h, W["norm"], c.norm_eps))
        print(f"  {name}: token {i + 1} of {len(tokens)} ({time.time() - t0:.0f} s)", flush=True)
    exact = np.stack(rows)
    np.savez_compressed(HERE / f"exact_{name}.npz", lead=exact[:, :cases.LOGIT_SUBSET],
                        strided=exact[:, ::cases.LOGIT_STRIDE],
                        top_values=np.take_along_axis(exact, golden["top_ids"], axis=1))
    reference = golden["strided"].astype(np.float64)
    err = np.abs(reference - exact[:, ::cases.LOGIT_STRIDE])
    return f"reference vs exact: max {err.max():.3g}"


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--only", nargs="*", default=["nano17_window", "lite", "lighting", "heavy"])
    args = parser.parse_args(argv)
    for name in args.only:
        t0 = time.time()
        print(f"exact_{name}: {run(name)} ({time.time() - t0:.1f}s)", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
