"""The failure path: a bounded device wait that runs out (reference contract:
a failed step latches the model until reset(), miracle_reasoning/model.py:
298-311).

No GPU is faulted.  The failure is made on the host's side: the model is
told (mr_model_inject_fault) not to publish one phase's words (the decode
kernel) or not to count its key / value rows (Heavy Medium's attention), so
the readers of that data wait until the short limit set with
mr_model_set_wait_limit, record the error and return; the context stays
usable.  Each case checks the error code (MR_ERR_TIMEOUT) and how fast it
came, that every later call raises until reset(), and that after reset() the
model computes exactly what a healthy model computes.
"""
import time

import numpy as np
import pytest

import cases
from conftest import submodule

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000  # 50 ms


def _fail_and_recover(model, prompt):
    native = submodule("_native")
    want = model.prefill(prompt, return_all=True)
    model.reset()
    native.call("mr_model_set_wait_limit", model._handle, LIMIT_NS)
    native.call("mr_model_inject_fault", model._handle, 0)
    t0 = time.perf_counter()
    with pytest.raises(native.CUDAError) as failure:
        model.prefill(prompt)
    assert failure.value.code == native.MR_ERR_TIMEOUT, failure.value
    assert "timed out" in str(failure.value) or "within" in str(failure.value)
    assert time.perf_counter() - t0 < 30.0  # the limit, not a hang
    # latched: every later call raises until reset() (model.py:298-299)
    with pytest.raises(RuntimeError, match="reset"):
        model.decode(int(prompt[0]))
    with pytest.raises(RuntimeError, match="reset"):
        model.prefill(prompt)
    # reset() clears the latch; without the fault the model is healthy again, bit for bit
    native.call("mr_model_inject_fault", model._handle, -1)
    model.reset()
    np.testing.assert_array_equal(model.prefill(prompt, return_all=True), want)
    assert model.position == len(prompt)


def test_decode_kernel_wait_times_out_latches_and_recovers(backend):
    config = cases.micro_config("nano15")
    model = submodule("model").MiracleModel(config, cases.micro_weights(config), backend=backend, context_length=32)
    _fail_and_recover(model, cases.micro_prompt("nano15"))


def test_heavy_medium_wait_times_out_latches_and_recovers(backend):
    config = cases.micro_config("heavy_mid")
    model = submodule("model").MiracleModel(config, cases.micro_weights(config), backend=backend,
                                            context_length=cases.micro_context("heavy_mid"))
    _fail_and_recover(model, cases.micro_prompt("heavy_mid")[:20])


def test_wait_limit_and_fault_arguments_are_checked(backend):
    native = submodule("_native")
    config = cases.micro_config("nano15")
    model = submodule("model").MiracleModel(config, cases.micro_weights(config), backend=backend, context_length=32)
    with pytest.raises(native.CUDAError, match="1 ms"):
        native.call("mr_model_set_wait_limit", model._handle, 1000)
    with pytest.raises(native.CUDAError, match="phase"):
        native.call("mr_model_inject_fault", model._handle, 10_000)
    with pytest.raises(native.CUDAError, match="phase"):
        native.call("mr_model_inject_fault", model._handle, -2)
