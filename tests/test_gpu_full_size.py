"""Every BASELINE configuration at its full architecture against the reference.

The fixtures (tests/golden/bench_*.npz, made by tests/golden/make_golden.py)
hold what the reference's own model.py computed, over its own kernels.cl, for
the same synthetic weights the device builds in HBM (the counter-hash
generator gives identical bits on the host and the device) and the same
prompt: per step (the prompt's last token, then each greedy decode step) the
leading 1024 logits, every 16th logit, the top 64 ids and values, the greedy
ids; for Heavy Medium also the routed experts, their weights and the kept
global blocks of all 64 (layer, inner loop) steps of every token.

* nano17_window: flashnano-1.7 with a 520-token prompt, which wraps the
  512-row local rings (batched tensor-core prefill);
* lite: flashlite-2.0, context 8192, a 16-token prompt (batched prefill);
* lighting: flashlighting-2.0 (YaRN factor 4 over a 4096 base, latent 512,
  window 2048), an 8-token prompt (batched prefill);
* heavy: heavy-medium-2.0 (36.5B parameters: hidden 4096, 32 layers, 64
  routed experts in 8 groups + 2 shared, two inner loops), a 4-token prompt.

Tolerance (north star: atol 2e-5, rtol 2e-4, the reference's own parity
tolerance, tests/test_inference.py:38).  At these depths and widths the
reference's float32 logits are themselves up to ~5e-5 from the exact values
(tests/golden/exact_*.npz: the same computation in float64, made by
tests/golden/make_exact.py), so the logits are checked twice:

* against the exact values at atol 2e-5, rtol 2e-4;
* against the reference at rtol 2e-4 and atol 2e-5 plus the reference's own
  largest deviation from the exact values on that fixture.

Greedy ids must equal the reference's (a step whose reference top-2 gap is
inside the tolerance is a near-tie, teacher-forced and counted); routing and
kept blocks exactly, expert weights (float outputs) at the parity tolerance.
"""
import json

import numpy as np
import pytest

import cases
from conftest import submodule

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-5, 2e-4


def _near_tie(top_values):
    return top_values[0] - top_values[1] <= ATOL + RTOL * abs(top_values[0])


def _run(backend, name, record=False):
    golden = np.load(cases.GOLDEN_DIR / f"bench_{name}.npz")
    config, stored, ctx, prompt, steps = cases.bench_case(name)
    assert prompt == golden["prompt"].tolist()
    model = submodule("model").MiracleModel.synthetic(config, stored=stored, backend=backend, context_length=ctx,
                                                      record_decisions=record)
    rows, ties = [model.prefill(prompt)], 0
    decisions = [model.decisions[-1]] if record else []
    for i in range(steps):
        want = int(golden["tokens"][i])
        got = int(np.argmax(rows[-1]))
        if got != want:
            assert _near_tie(golden["top_values"][i]), f"{name}: greedy step {i}: {got} != {want}"
            ties += 1
        rows.append(model.decode(want))
        if record:
            decisions.append(model.decisions[-1])
    logits = np.stack(rows)
    exact = np.load(cases.GOLDEN_DIR / f"exact_{name}.npz")
    views = {"lead": logits[:, :cases.LOGIT_SUBSET], "strided": logits[:, ::cases.LOGIT_STRIDE],
             "top_values": np.take_along_axis(logits, golden["top_ids"], axis=1)}
    reference_error = max(float(np.abs(golden[k] - exact[k]).max()) for k in views)
    for key, got in views.items():
        np.testing.assert_allclose(got, exact[key], atol=ATOL, rtol=RTOL, err_msg=f"{name} {key} vs exact")
        np.testing.assert_allclose(got, golden[key], atol=ATOL + reference_error, rtol=RTOL,
                                   err_msg=f"{name} {key} vs reference")
    return golden, model, decisions, ties


@pytest.mark.parametrize("name", ["nano17_window", "lite", "lighting"])
def test_full_architecture_matches_reference(backend, name):
    golden, model, _, ties = _run(backend, name)
    config, _, _, prompt, steps = cases.bench_case(name)
    assert model.position == len(prompt) + steps
    assert ties == 0
    if name == "nano17_window":  # the local rings wrapped: 512 rows kept, the oldest overwritten
        local = next(s for layer, s in enumerate(model.states) if config.layer_window(layer))
        assert local["ring"].length == 512 and local["ring"].count == len(prompt) + steps


def test_full_heavy_medium_matches_reference(backend):
    golden, model, decisions, ties = _run(backend, "heavy", record=True)
    config, _, _, prompt, _ = cases.bench_case("heavy")
    want = json.loads(str(golden["meta"]))["decisions"][len(prompt) - 1:]  # from the prompt's last token on
    assert ties == 0 and len(decisions) == len(want)
    for step, (mine, ref) in enumerate(zip(decisions, want)):
        experts = [loop for layer in mine for loop in layer["experts"]]
        weights = [loop for layer in mine for loop in layer["expert_weights"]]
        topk = [loop for layer in mine for loop in layer["topk"]]
        assert len(experts) == 64 and experts == ref["experts"], step
        assert topk == ref["topk"], step
        for got, exp in zip(weights, ref["expert_weights"]):
            np.testing.assert_allclose(got, exp, atol=ATOL, rtol=RTOL)
