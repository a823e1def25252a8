"""FlashLighting 2.0 on the decode engine (no memory slots: the latent cache
drops its oldest row, kept as a key/value ring of `window` rows) against the
CPU oracle, which recomputes every key and value from the stored latents each
step as the reference does (miracle_reasoning/model.py:146-190).

The case is large enough that the ring wraps (prompt longer than the window)
and attention splits the window into several key chunks merged across CTAs;
weights are BF16 with non-trivial gates.  Logits at the reference's own
tolerance (atol 2e-5, rtol 2e-4), greedy ids exact.
"""
import numpy as np
import pytest

import cases
from conftest import submodule
from oracle.host_backend import HostBackend
from oracle.reference_model import ReferenceModel

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-5, 2e-4


def _case():
    config = cases.ModelConfig(family="flashlighting-2.0", vocab_size=300, hidden_size=256, layers=2,
                               query_heads=4, kv_heads=4, head_dim=64, ffn_dim=384, max_positions=256,
                               window=100, latent_dim=64, memory_slots=0, residual_scale=0.5,
                               source={"rope_scaling_type": "yarn", "rope_scaling_factor": 2.0,
                                       "max_position_embeddings": 64})
    weights = cases.synthetic.synthetic_weights(config, "BF16", seed=5)
    for layer in range(config.layers):
        weights[f"layers.{layer}.attention_gate"] = np.full((1,), 0.7, np.float32)
        weights[f"layers.{layer}.ffn_gate"] = np.full((1,), 1.2, np.float32)
    prompt = cases.synthetic.prompt_ids(config.vocab_size, 150, seed=9).tolist()
    return config, weights, prompt


def test_lighting_ring_engine_matches_oracle(backend):
    config, weights, prompt = _case()
    model = submodule("model").MiracleModel(config, weights, backend=backend, context_length=200)
    oracle = ReferenceModel(config, weights, backend=HostBackend("oracle"), context_length=200)
    got = model.prefill(prompt, return_all=True)
    want = oracle.prefill(prompt, return_all=True)
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
    # the cache state the reference exposes after compaction
    state = model.states[0]
    assert state["latent"].shape == (config.window, config.latent_dim)
    assert state["positions"] == list(range(len(prompt) - config.window, len(prompt)))
    assert state["memory_size"] == 0 and state["counts"] == [1.0] * config.window
    assert oracle.states[0]["positions"] == state["positions"]
    # greedy continuation, device loop vs the oracle's
    ids = model.generate(prompt[:20], max_new_tokens=8)
    assert ids == oracle.generate(prompt[:20], max_new_tokens=8)


def test_lighting_batched_prefill_matches_token_by_token(backend):
    """The tensor-core prompt path (q | latent and gate | up GEMMs, latent_norm ->
    k | v GEMM, causal attention over ring + chunk) against the decode kernel
    run token by token, on a prompt longer than the window."""
    import ctypes as C
    config, weights, prompt = _case()
    native = submodule("_native")
    model = submodule("model").MiracleModel(config, weights, backend=backend, context_length=200)
    available = C.c_int(0)
    native.call("mr_model_set_batched_prefill", model._handle, 1, C.byref(available))
    assert available.value == 1
    batched = model.prefill(prompt, return_all=True)
    model.reset()
    native.call("mr_model_set_batched_prefill", model._handle, 0, C.byref(available))
    serial = model.prefill(prompt, return_all=True)
    np.testing.assert_allclose(batched, serial, atol=ATOL, rtol=RTOL)
    # decoding on from the batched prompt's ring gives the serial path's next logits
    model.reset()
    native.call("mr_model_set_batched_prefill", model._handle, 1, C.byref(available))
    model.prefill(prompt)
    np.testing.assert_allclose(model.decode(7), _serial_next(config, weights, prompt, backend), atol=ATOL, rtol=RTOL)


def _serial_next(config, weights, prompt, backend):
    import ctypes as C
    model = submodule("model").MiracleModel(config, weights, backend=backend, context_length=200)
    available = C.c_int(0)
    submodule("_native").call("mr_model_set_batched_prefill", model._handle, 0, C.byref(available))
    model.prefill(prompt)
    return model.decode(7)
