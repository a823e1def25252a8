"""Batched prefill (tensor-core GEMMs + causal attention over the chunk) against
the reference's outputs on BF16 models, and against the token-serial path.

The fixtures come from the reference itself (tests/golden/make_golden.py,
``prefill_<case>.npz``): a 48-token prompt that wraps the local window of the
micro architectures many times, the same prompt in two chunks, and greedy
decode steps that read the keys and values the prefill left in the rings.
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np
import pytest

import cases
from conftest import submodule

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-5, 2e-4  # the reference's parity tolerance (tests/test_inference.py:38)


def _model(backend, name, batched=True):
    config = cases.prefill_config(name)
    weights_mod = submodule("weights")
    weights = {k: (weights_mod.BF16Array(v) if v.dtype == np.uint16 else v)
               for k, v in cases.prefill_weights(config).items()}
    model = submodule("model").MiracleModel(config, weights, backend=backend, context_length=cases.PREFILL_CONTEXT)
    available = C.c_int(0)
    submodule("_native").call("mr_model_set_batched_prefill", model._handle, int(batched), C.byref(available))
    assert available.value == 1  # BF16 matrices, 16-byte rows: the batched path applies
    return model


@pytest.mark.parametrize("name", cases.PREFILL_CASES)
def test_batched_prefill_matches_reference(backend, name):
    golden = np.load(cases.GOLDEN_DIR / f"prefill_{name}.npz")
    meta = json.loads(str(golden["meta"]))
    model = _model(backend, name)
    prompt = cases.prefill_prompt(name)
    logits = model.prefill(prompt, return_all=True)
    np.testing.assert_allclose(logits, golden["logits"], atol=ATOL, rtol=RTOL)
    for layer, want in zip(model.states, meta["state"]):
        r = layer["ring"]
        assert [r.count, r.length, r.start, r.capacity] == want["ring"]
    # decode after the batched prompt reads the keys / values it appended
    steps = []
    for t in golden["tokens"]:
        steps.append(model.decode(int(t)))
    np.testing.assert_allclose(np.stack(steps), golden["steps"], atol=ATOL, rtol=RTOL)
    # last-token-only prefill returns the same final row
    model.reset()
    np.testing.assert_array_equal(model.prefill(prompt), logits[-1])


@pytest.mark.parametrize("name", cases.PREFILL_CASES)
def test_batched_prefill_in_chunks(backend, name):
    golden = np.load(cases.GOLDEN_DIR / f"prefill_{name}.npz")
    model = _model(backend, name)
    prompt = cases.prefill_prompt(name)
    split = cases.PREFILL_SPLIT
    chunked = np.concatenate([model.prefill(prompt[:split], return_all=True),
                              model.prefill(prompt[split:], return_all=True)])
    np.testing.assert_allclose(chunked, golden["chunked"], atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", cases.PREFILL_CASES)
def test_batched_and_token_serial_prefill_agree(backend, name):
    prompt = cases.prefill_prompt(name)
    batched = _model(backend, name, batched=True).prefill(prompt, return_all=True)
    serial = _model(backend, name, batched=False).prefill(prompt, return_all=True)
    np.testing.assert_allclose(batched, serial, atol=2 * ATOL, rtol=2 * RTOL)


def test_batched_prefill_full_size_nano17(backend):
    """BASELINE config 1 at full size: a 600-token prompt (two chunks, the local
    window wrapped) batched against token by token through the decode kernel."""
    config = submodule("synthetic").config_for("nano17")
    MiracleModel = submodule("model").MiracleModel
    prompt = submodule("synthetic").prompt_ids(config.vocab_size, 600).tolist()
    outs = []
    for batched in (True, False):
        model = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=2048)
        submodule("_native").call("mr_model_set_batched_prefill", model._handle, int(batched), None)
        logits = model.prefill(prompt, return_all=True)
        nxt = model.decode(int(np.argmax(logits[-1])))
        outs.append((logits, nxt))
        del model
    (lb, nb), (ls, ns) = outs
    scale = float(np.abs(ls).max())
    np.testing.assert_allclose(lb, ls, atol=4 * ATOL * max(1.0, scale), rtol=4 * RTOL)
    np.testing.assert_allclose(nb, ns, atol=4 * ATOL * max(1.0, scale), rtol=4 * RTOL)


def test_tcgen05_and_mma_sync_gemms_agree(backend):
    """The prefill's tcgen05 GEMMs against the mma.sync baseline kernel on a
    full-size nano-1.7 prompt (both sum the same exact BF16 products in FP32)."""
    config = submodule("synthetic").config_for("nano17")
    MiracleModel = submodule("model").MiracleModel
    prompt = submodule("synthetic").prompt_ids(config.vocab_size, 300).tolist()
    outs = []
    for mode in (1, 2):
        model = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=1024)
        submodule("_native").call("mr_model_set_batched_prefill", model._handle, mode, None)
        outs.append(model.prefill(prompt, return_all=True))
        del model
    scale = float(np.abs(outs[1]).max())
    np.testing.assert_allclose(outs[0], outs[1], atol=2 * ATOL * max(1.0, scale), rtol=2 * RTOL)


def test_batched_prompt_greedy_continuation_full_size(backend):
    """The greedy ids after a batched full-size prompt are those after the same prompt
    token by token (the batched GEMMs sum in another order: counted flips must be zero
    on this workload; nano-1.7, 600 tokens, the local window wrapped, 24 greedy steps)."""
    config = submodule("synthetic").config_for("nano17")
    MiracleModel = submodule("model").MiracleModel
    prompt = submodule("synthetic").prompt_ids(config.vocab_size, 600).tolist()
    runs = []
    for batched in (1, 0):
        model = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=1024)
        submodule("_native").call("mr_model_set_batched_prefill", model._handle, batched, None)
        logits, ids = model.prefill(prompt), []
        for _ in range(24):
            ids.append(int(np.argmax(logits)))
            logits = model.decode(ids[-1])
        runs.append(ids)
        del model
    flips = sum(a != b for a, b in zip(*runs))
    assert flips == 0, runs
