"""Parity case definitions shared by the golden generator and the tests.

Each case is rebuilt from this file wherever it runs (here, or on a GPU box
without the reference checkout); only the reference's OUTPUTS live in the
committed fixtures.

Micro cases follow the reference's own fixtures: the ``tiny()`` model of
tests/test_inference.py:15-22 (vocab 32, hidden 16, 2 layers, 4 query / 2 KV
heads, head_dim 4, ffn 24, window 4, global layer 2, matrices N(0, 0.05) from
``default_rng(72)``, 1-D tensors 1.0) and the per-family micro configurations
of tests/make_reference.py:19-73 (CBR chunk 3 / 2 slots; global KV heads 4;
latent 8 with 2 memory slots and gates 0.7 / 1.2; MoE with 4 routed + 1 shared
expert, 2 groups, top-k 1..2, block 3, 2 global slots).  The prompt is
make_reference.py:84's id list.
"""
from __future__ import annotations

import importlib
import sys
from dataclasses import replace  # noqa: F401  (re-exported)
from pathlib import Path

import numpy as np

_REPO = Path(__file__).resolve().parents[2]
if str(_REPO) not in sys.path:
    sys.path.insert(0, str(_REPO))
PKG = importlib.import_module("miraclereasoning-cpu_b200")
ModelConfig = PKG.config.ModelConfig
expected_shapes = PKG.weights.expected_shapes
synthetic = importlib.import_module("miraclereasoning-cpu_b200.synthetic")

GOLDEN_DIR = Path(__file__).resolve().parent
PROMPT = [1, 5, 3, 7, 11, 9, 4, 17, 8, 6, 10, 12]


def _tiny_base(family, **changes):
    base = dict(family=family, vocab_size=32, hidden_size=16, layers=2, query_heads=4, kv_heads=2,
                head_dim=4, ffn_dim=24, max_positions=32, window=4, global_layers=(2,))
    base.update(changes)
    return ModelConfig(**base)


def _heavy_source(**changes):
    source = {"routed_experts": 4, "router_groups": 2, "router_top_k_max": 2, "router_top_k_min": 1,
              "shared_experts": 1,
              "long_context": {"local_window": 4, "global_block_size": 3, "global_slots": 2,
                               "target_context": 32}}
    source.update(changes)
    return source


def micro_config(name):
    if name == "nano15":
        return _tiny_base("flashnano-1.5")
    if name == "nano15_untied":
        return _tiny_base("flashnano-1.5", tie_embeddings=False)
    if name == "nano16":
        return _tiny_base("flashnano-1.6", cbr_chunk_size=3, cbr_slots=2)
    if name == "nano17":
        return _tiny_base("flashnano-1.7", global_kv_heads=4)
    if name == "lite":
        return _tiny_base("flashlite-2.0", residual_scale=0.5, window=None, global_layers=())
    if name == "lite_noqk":
        return _tiny_base("flashlite-2.0", qk_norm=False, rope_theta=5e5, residual_scale=0.5)
    if name == "lighting":
        return _tiny_base("flashlighting-2.0", global_layers=(), latent_dim=8, memory_slots=2,
                          residual_scale=0.5,
                          source={"rope_scaling_type": "yarn", "rope_scaling_factor": 2.0,
                                  "max_position_embeddings": 16})
    if name == "lighting_drop":
        return replace(micro_config("lighting"), memory_slots=0)
    if name == "heavy":
        return _tiny_base("heavy-medium-2.0", global_layers=(), latent_dim=8, ffn_dim=12,
                          inner_loop_steps=2, source=_heavy_source())
    if name == "heavy_mid":
        return ModelConfig(family="heavy-medium-2.0", vocab_size=64, hidden_size=64, layers=2,
                           query_heads=4, kv_heads=2, head_dim=16, ffn_dim=24, max_positions=96,
                           window=8, latent_dim=32, inner_loop_steps=2,
                           source=_heavy_source(routed_experts=16, router_groups=4, router_top_k_max=4,
                                                router_top_k_min=2, shared_experts=2,
                                                long_context={"local_window": 8, "global_block_size": 4,
                                                              "global_slots": 3, "target_context": 96}))
    raise KeyError(name)


MICRO_CASES = ("nano15", "nano15_untied", "nano16", "nano17", "lite", "lite_noqk", "lighting",
               "lighting_drop", "heavy", "heavy_mid")


def micro_weights(config, seed=72):
    """tiny()-style weights; lighting gates and heavy router biases made non-trivial."""
    rng = np.random.default_rng(seed)
    weights = {k: (rng.normal(0, 0.05, shape).astype(np.float32) if len(shape) == 2
                   else np.ones(shape, np.float32))
               for k, shape in expected_shapes(config).items()}
    extra = np.random.default_rng(seed + 1)
    for name in list(weights):
        if name.endswith("attention_gate"):
            weights[name] = np.full((1,), 0.7, np.float32)
        elif name.endswith("ffn_gate"):
            weights[name] = np.full((1,), 1.2, np.float32)
        elif ".router." in name and weights[name].ndim == 1:
            weights[name] = extra.normal(0, 0.3, weights[name].shape).astype(np.float32)
    if config.family == "heavy-medium-2.0":
        # Sharper routers so that routing decisions vary from token to token.
        for name in list(weights):
            if name.endswith(("router.coarse.weight", "router.fine.weight")):
                weights[name] = (weights[name] * np.float32(20)).astype(np.float32)
    return weights


def micro_prompt(name):
    if name == "heavy_mid":
        return np.random.default_rng(5).integers(0, 64, 80).tolist()
    return list(PROMPT)


def micro_context(name):
    return 96 if name == "heavy_mid" else 32


# Benchmark-shape cases: the real architectures, short token windows.
def bench_case(name):
    """(config, stored dtype, context, prompt ids, greedy decode steps).

    Every BASELINE configuration at its full architecture.  The context is the
    workload's wherever the reference's CPU run can hold its caches; Heavy
    Medium uses 2048 (the rings are context-sized, and nothing else depends on
    the context while every position fits).  ``nano17_window`` runs a prompt
    that crosses the 512-row local window, so the local rings wrap."""
    config = synthetic.config_for(name.split("_")[0])
    if name == "nano15":
        ctx, prompt_len, decode = synthetic.WORKLOADS["nano15"]
        return config, "F32", ctx, synthetic.prompt_ids(config.vocab_size, prompt_len).tolist(), decode
    sizes = {"nano17": (2048, 8, 4), "nano17_window": (2048, 520, 4), "lite": (8192, 16, 4),
             "lighting": (16384, 8, 4), "heavy": (2048, 4, 2)}
    if name not in sizes:
        raise KeyError(name)
    ctx, prompt_len, decode = sizes[name]
    return config, "BF16", ctx, synthetic.prompt_ids(config.vocab_size, prompt_len).tolist(), decode


BENCH_CASES = ("nano15", "nano17", "nano17_window", "lite", "lighting", "heavy")
LOGIT_SUBSET = 1024     # leading logits stored per step for wide vocabularies
LOGIT_STRIDE = 16       # and every 16th logit (the fixtures of the wide-vocabulary cases)
TOPK_STORED = 64


# Batched-prefill cases: the micro architectures with BF16 matrices (the
# engine's tensor-core prefill applies to BF16 models) and a prompt long enough
# to wrap the local window several times.
PREFILL_CASES = ("nano17", "lite")
PREFILL_CONTEXT = 96
PREFILL_SPLIT = 13


def prefill_config(name):
    return replace(micro_config(name), max_positions=PREFILL_CONTEXT)


def prefill_prompt(name):
    return np.random.default_rng(11).integers(0, prefill_config(name).vocab_size, 48).tolist()


def bf16_bits(array):
    """Round-to-nearest-even BF16 bits of a float32 array."""
    bits = np.ascontiguousarray(array, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


def prefill_weights(config):
    """micro_weights with every matrix stored as BF16 (uint16 bits); 1-D tensors stay float32."""
    return {k: (bf16_bits(v) if v.ndim == 2 else v) for k, v in micro_weights(config).items()}


def widen_bf16(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)
