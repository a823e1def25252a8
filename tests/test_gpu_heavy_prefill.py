"""Heavy Medium batched prompt (csrc/heavy_prefill.cuh) against the token step.

The reference runs a prompt token by token (model.py:295-312); the batched
path must leave the same sequence state and give the same logits within the
parity tolerance: every token's logits, the last token's kept blocks and
experts, and the decode steps that continue from the rows, block means and
running block sums the chunk left.  The micro case is heavy_mid with its
matrices rounded to BF16 (the batched path needs BF16 weights); the prompt
wraps the 8-row window ten times and fills 20 blocks of 4 rows, and the
chunked form starts its second chunk inside a block.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import cases
from conftest import submodule

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-5, 2e-4  # the reference's parity tolerance (tests/test_inference.py:38)


def _bf16_weights(config):
    weights_mod = submodule("weights")
    out = {}
    for name, value in cases.micro_weights(config).items():
        out[name] = weights_mod.BF16Array(weights_mod.float32_to_bf16_bits(value)) if value.ndim == 2 else value
    return out


def _model(backend, batched, record=False):
    config = cases.micro_config("heavy_mid")
    model = submodule("model").MiracleModel(config, _bf16_weights(config), backend=backend,
                                            context_length=cases.micro_context("heavy_mid"),
                                            record_decisions=record)
    available = C.c_int(0)
    submodule("_native").call("mr_model_set_batched_prefill", model._handle, int(batched), C.byref(available))
    assert available.value == 1  # BF16 matrices with 16-byte rows, one GPU: the batched path applies
    return model


def _continue(model, logits, steps=4):
    out, token = [], int(np.argmax(logits))
    for _ in range(steps):
        row = model.decode(token)
        out.append(row)
        token = int(np.argmax(row))
    return np.stack(out)


def test_batched_prompt_matches_token_step(backend):
    prompt = cases.micro_prompt("heavy_mid")
    batched, serial = _model(backend, True), _model(backend, False)
    lb = batched.prefill(prompt, return_all=True)
    ls = serial.prefill(prompt, return_all=True)
    np.testing.assert_allclose(lb, ls, atol=2 * ATOL, rtol=2 * RTOL)
    assert batched.position == serial.position == len(prompt)
    # the last token's decisions, where the token step leaves its own
    batched._read_decisions()
    serial._read_decisions()
    for got, want in zip(batched._decisions[-1], serial._decisions[-1]):
        assert got["topk"] == want["topk"] and got["experts"] == want["experts"]
        for gw, ww in zip(got["expert_weights"], want["expert_weights"]):  # float32 values, not decisions
            np.testing.assert_allclose(gw, ww, atol=ATOL, rtol=RTOL)
    # decode continues from the rows, block means and running sums the chunk left
    np.testing.assert_allclose(_continue(batched, lb[-1]), _continue(serial, ls[-1]), atol=2 * ATOL, rtol=2 * RTOL)


def test_batched_prompt_in_chunks(backend):
    """Two chunks, the second starting inside a block (13 % 4 = 1): the carried
    running block sums and the earlier chunk's rows are what it reads."""
    prompt = cases.micro_prompt("heavy_mid")
    chunked = _model(backend, True)
    parts = np.concatenate([chunked.prefill(prompt[:13], return_all=True),
                            chunked.prefill(prompt[13:], return_all=True)])
    serial = _model(backend, False)
    ls = serial.prefill(prompt, return_all=True)
    np.testing.assert_allclose(parts, ls, atol=2 * ATOL, rtol=2 * RTOL)
    np.testing.assert_allclose(_continue(chunked, parts[-1]), _continue(serial, ls[-1]), atol=2 * ATOL, rtol=2 * RTOL)


def test_last_row_only_equals_all_rows(backend):
    prompt = cases.micro_prompt("heavy_mid")
    model = _model(backend, True)
    rows = model.prefill(prompt, return_all=True)
    model.reset()
    np.testing.assert_array_equal(model.prefill(prompt), rows[-1])


def test_batched_prompt_full_size(backend):
    """heavy-medium-2.0 at full size: a 300-token prompt (five blocks of 64) batched
    against token by token.

    Over 300 tokens x 64 layer-loops the router ranks 64 experts 19,200 times;
    the batched router GEMM sums the same exact products in another order, so
    where two experts' probabilities tie to within rounding the two paths may
    rank them differently (the reference's own float32 order is a third one).
    Such a swap changes that token's expert and, through its keys and values,
    later tokens slightly.  The test therefore holds every row up to the first
    token whose decisions differ to the parity tolerance, requires that token's
    difference to be a swap of two experts whose normalised weights agree to
    float32 rounding (a tie, not a wrong computation), and requires the kept
    blocks to agree there."""
    config = submodule("synthetic").config_for("heavy")
    model = submodule("model").MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=2048,
                                                      record_decisions=True)
    prompt = submodule("synthetic").prompt_ids(config.vocab_size, 300).tolist()
    native = submodule("_native")
    ls = model.prefill(prompt, return_all=True)  # token by token: every token's decisions recorded
    serial_decisions = model.decisions
    model.record_decisions = False
    model.reset()
    native.call("mr_model_set_batched_prefill", model._handle, 1, None)
    lb = model.prefill(prompt, return_all=True)
    scale = max(1.0, float(np.abs(ls).max()))
    atol = 4 * ATOL * scale
    bad = np.nonzero(~np.all(np.isclose(lb, ls, atol=atol, rtol=4 * RTOL), axis=1))[0]
    first = int(bad[0]) if len(bad) else len(prompt)
    np.testing.assert_allclose(lb[:first], ls[:first], atol=atol, rtol=4 * RTOL)
    if first == len(prompt):
        return
    # the earliest token whose decisions differ (at or a few tokens before that row): the
    # batched decisions of token n from a batched prompt ending at n (the chunk is causal)
    for n in range(max(0, first - 8), first + 1):
        model.reset()
        model.prefill(prompt[:n + 1])
        model._decisions = []
        model._read_decisions()
        got_token, want_token = model._decisions[-1], serial_decisions[n]
        if all(g["topk"] == w["topk"] and g["experts"] == w["experts"] for g, w in zip(got_token, want_token)):
            continue
        # the first decision in execution order (layer, then inner loop) that differs must be a
        # tie: the same kept blocks, experts swapped at one rank, every weight equal to rounding
        # (what follows it in later layers is its consequence, not a separate event)
        for layer, (got, want) in enumerate(zip(got_token, want_token)):
            for loop in range(len(got["experts"])):
                same = got["topk"][loop] == want["topk"][loop] and got["experts"][loop] == want["experts"][loop]
                if same:
                    continue
                assert got["topk"][loop] == want["topk"][loop], f"token {n} layer {layer}: kept blocks differ"
                ge, we = got["experts"][loop], want["experts"][loop]
                assert len(ge) == len(we) and sum(a != b for a, b in zip(ge, we)) >= 1
                np.testing.assert_allclose(got["expert_weights"][loop], want["expert_weights"][loop], rtol=1e-4)
                return
    raise AssertionError(f"row {first} differs but no token from {max(0, first - 8)} on routes differently")
