"""Heavy Medium 2.0 on the device token step (csrc/heavy.cu) against the CPU
oracle, which runs the reference's own control flow with the top-k and the
routing in float32 NumPy (miracle_reasoning/model.py:192-255).

Sized so that the decisions matter: more global blocks than top-k slots (the
distance penalty and stable ordering pick the kept blocks), a local window
shorter than the history, 16 routed experts in 4 groups with an adaptive
top-k of 2..4 plus 2 shared experts, two inner loops; BF16 weights with
router biases made non-uniform.  Logits at the reference's tolerance
(atol 2e-5, rtol 2e-4); kept blocks and experts per token exactly.
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
    config = cases.ModelConfig(
        family="heavy-medium-2.0", vocab_size=200, hidden_size=128, layers=2, query_heads=4, kv_heads=2,
        head_dim=32, ffn_dim=64, max_positions=128, window=16, latent_dim=32, inner_loop_steps=2,
        source={"routed_experts": 16, "router_groups": 4, "router_top_k_max": 4, "router_top_k_min": 2,
                "shared_experts": 2,
                "long_context": {"local_window": 16, "global_block_size": 8, "global_slots": 3,
                                 "target_context": 128}})
    weights = cases.synthetic.synthetic_weights(config, "BF16", seed=11)
    rng = np.random.default_rng(3)
    for name in list(weights):
        if "bias" in name:
            weights[name] = rng.normal(0, 2.5, np.shape(weights[name])).astype(np.float32)
    prompt = cases.synthetic.prompt_ids(config.vocab_size, 90, seed=4).tolist()
    return config, weights, prompt


def _oracle_decisions(oracle):
    out = []
    for token in oracle.decisions:
        entry = {"topk": [], "experts": []}
        for layer in token:
            entry["topk"].extend(layer.get("topk_blocks", []))
            entry["experts"].extend(layer.get("experts", []))
        out.append(entry)
    return out


def test_heavy_device_step_matches_oracle(backend):
    config, weights, prompt = _case()
    model = submodule("model").MiracleModel(config, weights, backend=backend, context_length=120,
                                            record_decisions=True)
    oracle = ReferenceModel(config, weights, backend=HostBackend("oracle"), context_length=120, record=True)
    got = model.prefill(prompt, return_all=True)
    want = oracle.prefill(prompt, return_all=True)
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
    expected = _oracle_decisions(oracle)
    assert len(model.decisions) == len(expected) == len(prompt)
    masked = False
    for token, (mine, ref) in enumerate(zip(model.decisions, expected)):
        topk = [loop for layer in mine for loop in layer["topk"]]
        experts = [loop for layer in mine for loop in layer["experts"]]
        assert topk == ref["topk"], token
        assert experts == ref["experts"], token
        masked = masked or any(len(head) == 3 and token >= 24 for loop in topk for head in loop)
    assert masked  # the top-k did choose among more blocks than slots
    # the device path without per-token reads: the token step gives the same logits bit for
    # bit, the batched prompt (tcgen05 GEMMs, another summation order) within the tolerance
    fast = submodule("model").MiracleModel(config, weights, backend=backend, context_length=120)
    native = submodule("_native")
    native.call("mr_model_set_batched_prefill", fast._handle, 0, None)
    np.testing.assert_array_equal(fast.prefill(prompt, return_all=True), got)
    fast.reset()
    native.call("mr_model_set_batched_prefill", fast._handle, 1, None)
    np.testing.assert_allclose(fast.prefill(prompt, return_all=True), got, atol=ATOL, rtol=RTOL)
    fast.reset()
    # greedy continuation matches the oracle's
    assert fast.generate(prompt[:30], max_new_tokens=8) == oracle.generate(prompt[:30], max_new_tokens=8)
