"""Pin the CPU oracle before trusting it (no GPU).

1. The plain-C restatement (oracle/kernels.c) is bit-identical to the
   reference's own kernels.cl compiled for the host (oracle/_ref) on random
   inputs for all thirteen kernels, and reproduces the reference's known-answer
   cases (tests/test_opencl.py:19-63 shapes and seeds, stored in kernels.npz).
2. The restated token loop (oracle/reference_model.py) driven by the C kernels
   reproduces, bit for bit, every output the reference itself produced in
   tests/golden: logits, chunked prefill, cache state, heavy top-k blocks, MoE
   experts, latent positions, greedy and sampled generation.
"""
import json

import numpy as np
import pytest

import cases
from oracle.host_backend import HostBackend, SIGNATURES, load_kernels
from oracle.reference_model import ReferenceModel

GOLDEN = cases.GOLDEN_DIR


def _random_args(name, rng):
    """Random, in-bounds arguments for one NDRange of kernel ``name``."""
    f = lambda *shape: rng.normal(size=shape).astype(np.float32)  # noqa: E731
    if name == "linear":
        rows, out, inner = 3, 37, 45
        return (out, rows), [f(rows, inner), f(out, inner), np.zeros(rows * out, np.float32), rows, out, inner]
    if name == "rms":
        return (5,), [f(5, 33), f(33), np.zeros(5 * 33, np.float32), 5, 33, np.float32(1e-6), 1]
    if name == "rope":
        rows, heads, dim = 3, 4, 10
        return (rows * heads * dim // 2,), [f(rows, heads * dim), np.abs(f(dim // 2)),
                                           np.array([7, 300, 32767], np.float32),
                                           np.zeros(rows * heads * dim, np.float32), rows, heads, dim, 1]
    if name == "swiglu":
        return (50,), [f(50) * 4, f(50), np.zeros(50, np.float32), 50]
    if name == "axpy":
        return (50,), [f(50), f(50), np.zeros(50, np.float32), 50, np.float32(0.37)]
    if name in ("scores", "mix"):
        heads, kvh, dim, cap, start, length, extra = 6, 2, 8, 7, 5, 6, 3
        q = f(heads * dim)
        keys, extra_k = f(cap, kvh * dim), f(extra, kvh * dim)
        if name == "scores":
            return (length + extra, heads), [q, keys, extra_k, np.zeros(heads * (length + extra), np.float32),
                                             heads, kvh, dim, cap, start, length, extra]
        p = np.abs(f(heads, length + extra))
        return (heads * dim,), [p, keys, extra_k, np.zeros(heads * dim, np.float32), heads, kvh, dim, cap,
                                start, length, extra]
    if name == "softmax":
        return (4,), [f(4, 21) * 30, np.zeros(84, np.float32), 4, 21]
    if name == "latent_mask":
        return (9, 3), [f(3, 9), np.arange(9, dtype=np.float32), 3, 9, 2, 5]
    if name == "pool_scores":
        return (5, 2), [f(5, 16), f(2, 16), np.zeros(10, np.float32), 5, 2, 16]
    if name == "pool_mix":
        return (16, 2), [f(5, 16), np.abs(f(2, 5)), np.zeros(32, np.float32), np.zeros(2, np.float32), 5, 2, 16, 11]
    if name == "merge_rows":
        return (12,), [f(2, 12), np.zeros(12, np.float32), 12, np.float32(3.0), np.float32(1.0)]
    if name == "block_means":
        return (8, 4), [f(11, 8), np.zeros(32, np.float32), 11, 8, 3]
    raise KeyError(name)


def _run(lib, prefix, name, shape, args):
    import ctypes as C
    arrays = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a for a in args]
    values = []
    for a in arrays:
        if isinstance(a, np.ndarray):
            values.append(C.c_void_p(a.ctypes.data))
        elif isinstance(a, (float, np.floating)):
            values.append(C.c_float(a))
        else:
            values.append(C.c_int(a))
    getattr(lib, prefix + name)(*shape, *values)
    return [a for a in arrays if isinstance(a, np.ndarray)]


@pytest.mark.parametrize("name", sorted(SIGNATURES))
def test_c_restatement_bit_identical_to_reference_kernels(name):
    try:
        ref_lib, ref_prefix = load_kernels("reference")
    except Exception as exc:  # the reference checkout and its prebuilt library are both absent
        pytest.skip(f"reference kernels unavailable: {exc}")
    ora_lib, ora_prefix = load_kernels("oracle")
    for seed in range(3):
        shape, args = _random_args(name, np.random.default_rng(seed))
        ref_out = _run(ref_lib, ref_prefix, name, shape, [a.copy() if isinstance(a, np.ndarray) else a for a in args])
        ora_out = _run(ora_lib, ora_prefix, name, shape, [a.copy() if isinstance(a, np.ndarray) else a for a in args])
        for r, o in zip(ref_out, ora_out):
            np.testing.assert_array_equal(r.view(np.uint32), o.view(np.uint32))


def test_oracle_kernel_known_answers():
    g = np.load(GOLDEN / "kernels.npz")
    b = HostBackend("oracle")
    np.testing.assert_array_equal(b.read(b.linear(b.upload(g["lin_x"]), b.upload(g["lin_w"]))), g["lin_y"])
    np.testing.assert_allclose(g["lin_y"], g["lin_x"] @ g["lin_w"].T, atol=4e-6)
    np.testing.assert_array_equal(b.read(b.norm(b.upload(g["lin_x"]), b.upload(g["rms_w"]), 19, 1e-6)), g["rms_y"])
    np.testing.assert_array_equal(b.read(b.softmax(b.upload(g["sm_x"]))), g["sm_y"])
    pos, freq = np.array([7, 29], np.float32), np.array([1, .1, .01], np.float32)
    for split in (0, 1):
        got = b.rotate(b.upload(g["rope_x"].reshape(2, 18)), b.upload(freq), b.upload(pos), 3, 6, bool(split))
        np.testing.assert_array_equal(b.read(got), g[f"rope_y{split}"])
    att = b.attention(b.upload(g["att_q"].reshape(1, -1)), b.upload(g["att_k"].reshape(5, -1)),
                      b.upload(g["att_v"].reshape(5, -1)), heads=4, kv_heads=2, dim=6, start=3, length=4,
                      extra_keys=b.upload(g["att_rk"].reshape(3, -1)),
                      extra_values=b.upload(g["att_rv"].reshape(3, -1)), extra_length=3)
    np.testing.assert_array_equal(b.read(att), g["att_y"])


def decisions_of(model):
    """Flatten the oracle's per-token decision records into the golden layout."""
    out = []
    for token in model.decisions:
        entry = {"topk": [], "experts": [], "expert_weights": [], "latent_positions": [], "memory_size": []}
        for layer in token:
            entry["topk"] += layer.get("topk_blocks", [])
            entry["experts"] += layer.get("experts", [])
            entry["expert_weights"] += layer.get("expert_weights", [])
            entry["latent_positions"] += layer.get("latent_positions", [])
            entry["memory_size"] += layer.get("memory_size", [])
        out.append(entry)
    return out


@pytest.mark.parametrize("name", cases.MICRO_CASES)
def test_oracle_model_reproduces_reference_outputs(name):
    golden = np.load(GOLDEN / f"micro_{name}.npz")
    meta = json.loads(str(golden["meta"]))
    config = cases.micro_config(name)
    model = ReferenceModel(config, cases.micro_weights(config), backend=HostBackend("oracle"),
                           context_length=cases.micro_context(name), record=True)
    prompt = cases.micro_prompt(name)
    np.testing.assert_array_equal(model.prefill(prompt, return_all=True), golden["logits"])
    for got, want in zip(decisions_of(model), meta["decisions"]):
        assert got["topk"] == want["topk"]
        assert got["experts"] == want["experts"]
        np.testing.assert_array_equal(np.float32(sum(got["expert_weights"], [])),
                                      np.float32(sum(want["expert_weights"], [])))
        assert got["latent_positions"] == want["latent_positions"]
        assert got["memory_size"] == want["memory_size"]
    for layer, want in zip(model.states, meta["state"]):
        if "ring" in want:
            r = layer["ring"]
            assert [r.count, r.length, r.start, r.capacity] == want["ring"]
        if "relay" in want:
            assert layer["relay"].count == want["relay"]
        if "latent_rows" in want:
            assert layer["latent"].shape[0] == want["latent_rows"]
            assert layer["positions"] == want["positions"]
        if "loops" in want:
            assert [[s["ring"].count, s["ring"].capacity] for s in layer["loops"]] == want["loops"]
    model.reset()
    chunked = np.concatenate([model.prefill(prompt[:5], return_all=True), model.prefill(prompt[5:], return_all=True)])
    np.testing.assert_array_equal(chunked, golden["chunked"])
    assert model.generate(prompt[:3], max_new_tokens=6) == golden["greedy"].tolist()
    assert model.generate(prompt[:2], max_new_tokens=5, temperature=0.8, top_k=5, top_p=0.9,
                          seed=7) == golden["sampled"].tolist()


def test_oracle_bench_nano15_greedy_decode():
    golden = np.load(GOLDEN / "bench_nano15.npz")
    config, stored, ctx, prompt, steps = cases.bench_case("nano15")
    weights = cases.synthetic.synthetic_weights(config, stored)
    model = ReferenceModel(config, weights, backend=HostBackend("oracle"), context_length=ctx)
    logits = [model.prefill(prompt)]
    tokens = []
    for _ in range(steps):
        tokens.append(int(np.argmax(logits[-1])))
        logits.append(model.decode(tokens[-1]))
    assert tokens == golden["tokens"].tolist()
    np.testing.assert_array_equal(np.stack(logits), golden["full"])


@pytest.mark.parametrize("name", cases.PREFILL_CASES)
def test_oracle_prefill_bf16_cases(name):
    """The BF16 prefill fixtures (reference-generated) reproduced bit for bit."""
    golden = np.load(GOLDEN / f"prefill_{name}.npz")
    config = cases.prefill_config(name)
    weights = {k: (cases.widen_bf16(v) if v.dtype == np.uint16 else v) for k, v in cases.prefill_weights(config).items()}
    model = ReferenceModel(config, weights, backend=HostBackend("oracle"), context_length=cases.PREFILL_CONTEXT)
    prompt = cases.prefill_prompt(name)
    np.testing.assert_array_equal(model.prefill(prompt, return_all=True), golden["logits"])
    steps = [model.decode(int(t)) for t in golden["tokens"]]
    np.testing.assert_array_equal(np.stack(steps), golden["steps"])
