"""Sampled generate on the device (csrc/sampler.cu) against the reference's
host procedure (model.py:318-357 with sample_next, model.py:343-352): the same
seeded tokens, for every family path (the decode kernel, its batched prompt,
Heavy Medium's token step and batched prompt), several temperatures, top_k and
top_p, an early EOS, and the non-finite stop."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import cases
from conftest import submodule

pytestmark = pytest.mark.gpu

SETTINGS = [(0.8, 0, 1.0, 3), (1.0, 5, 1.0, 11), (0.7, 0, 0.9, 17), (1.3, 20, 0.8, 23), (2.0, 0, 0.5, 5)]


def _host_generate(model, prompt, max_new, temperature, top_k, top_p, seed, eos):
    """The reference's loop, sampling on the host (model.py:318-357)."""
    sample_next = submodule("model").sample_next
    model.reset()
    rng, out = np.random.default_rng(seed), []
    logits = model.prefill(prompt)
    for i in range(max_new):
        token = int(np.argmax(logits)) if temperature == 0 else sample_next(logits, temperature, top_k, top_p, rng)
        out.append(token)
        if token == eos or i + 1 == max_new:
            break
        logits = model.decode(token)
    return out


def _bf16(config, weights):
    wm = submodule("weights")
    return {k: (wm.BF16Array(wm.float32_to_bf16_bits(v)) if v.ndim == 2 else v) for k, v in weights.items()}


def _models(backend):
    Model = submodule("model").MiracleModel
    out = []
    for name in ("nano15", "heavy_mid"):
        config = cases.micro_config(name)
        weights = cases.micro_weights(config)
        ctx = cases.micro_context(name)
        out.append((name, Model(config, weights, backend=backend, context_length=ctx), cases.micro_prompt(name)[:12]))
        # BF16 matrices: the batched prompt paths
        out.append((name + "_bf16", Model(config, _bf16(config, weights), backend=backend, context_length=ctx),
                    cases.micro_prompt(name)[:12]))
    return out


@pytest.mark.parametrize("temperature,top_k,top_p,seed", SETTINGS)
def test_device_sampling_matches_host_procedure(backend, temperature, top_k, top_p, seed):
    for name, model, prompt in _models(backend):
        eos = model.config.eos_token_id
        want = _host_generate(model, prompt, 10, temperature, top_k, top_p, seed, eos)
        got = model.generate(prompt, max_new_tokens=10, temperature=temperature, top_k=top_k, top_p=top_p,
                             seed=seed, eos_token_id=eos)
        assert got == want, name
        assert model.position == len(prompt) + len(got) - 1
        # the sequence continues from the generated state like after host decoding
        nxt = model.decode(got[-1])
        model.reset()
        ref = _host_generate(model, prompt, len(got), temperature, top_k, top_p, seed, eos)
        np.testing.assert_array_equal(model.decode(ref[-1]), nxt)


def test_device_sampling_stops_at_eos(backend):
    name, model, prompt = _models(backend)[0]
    free = model.generate(prompt, max_new_tokens=12, temperature=1.5, seed=29)
    eos = free[4]  # a token the sequence produces: the generation must stop there
    stop = free.index(eos)
    got = model.generate(prompt, max_new_tokens=12, temperature=1.5, seed=29, eos_token_id=eos)
    assert got == free[:stop + 1]
    assert got == _host_generate(model, prompt, 12, 1.5, 0, 1.0, 29, eos)


def test_device_sampling_full_size_nano17(backend):
    """BASELINE config 1 at full size (32000 tokens to sort, batched prompt)."""
    config = submodule("synthetic").config_for("nano17")
    model = submodule("model").MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=256)
    prompt = submodule("synthetic").prompt_ids(config.vocab_size, 40).tolist()
    for temperature, top_k, top_p, seed in [(0.9, 0, 0.95, 7), (1.2, 50, 1.0, 8)]:
        want = _host_generate(model, prompt, 8, temperature, top_k, top_p, seed, config.eos_token_id)
        got = model.generate(prompt, max_new_tokens=8, temperature=temperature, top_k=top_k, top_p=top_p, seed=seed)
        assert got == want


def test_device_sampling_non_finite_logits_raise(backend):
    config = cases.micro_config("nano15")
    weights = cases.micro_weights(config)
    prompt = cases.micro_prompt("nano15")[:6]
    weights["embed"] = weights["embed"].copy()
    weights["embed"][prompt[-1], 0] = np.inf  # the last prompt token's row: non-finite logits
    model = submodule("model").MiracleModel(config, weights, backend=backend, context_length=32)
    with pytest.raises(FloatingPointError):
        model.generate(prompt, max_new_tokens=4, temperature=1.0, seed=3)
