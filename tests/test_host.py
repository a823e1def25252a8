"""Host-side logic without a GPU: config, weights I/O, synthetic models, C ABI.

Ports the reference's own non-device tests (tests/test_weights_config.py and
tests/test_inference.py:102-106) to this package and pins the config tables
against fixtures the reference produced (tests/golden/configs.npz).
"""
import ctypes
import dataclasses
import importlib
import json
import re
import struct
from dataclasses import replace

import numpy as np
import pytest

import cases
from conftest import REPO, submodule

configs_golden = np.load(cases.GOLDEN_DIR / "configs.npz")
CONFIG_META = json.loads(str(configs_golden["meta"]))


def _variant(name):
    if name.startswith("bench_"):
        return cases.synthetic.config_for(name[6:])
    if name in cases.MICRO_CASES:
        return cases.micro_config(name)
    return cases.PKG.config.ModelConfig.from_dict(CONFIG_META[name]["to_dict"])


@pytest.mark.parametrize("name", sorted(CONFIG_META))
def test_inverse_frequencies_and_name_tables_match_reference(pkg, name):
    config = _variant(name)
    np.testing.assert_array_equal(config.inverse_frequencies(), configs_golden[f"freq_{name}"])
    meta = CONFIG_META[name]
    assert pkg.weights.native_names(config) == meta["native_names"]
    assert {k: list(v) for k, v in pkg.weights.expected_shapes(config).items()} == meta["expected_shapes"]
    assert json.loads(json.dumps(config.to_dict())) == meta["to_dict"]


def test_safetensors_roundtrip_and_bfloat16_tiles(pkg, tmp_path):
    w = pkg.weights
    arrays = {"x": np.arange(21, dtype=np.float32).reshape(3, 7), "scale": np.ones(7, np.float32)}
    w.save_safetensors(tmp_path / "f32.safetensors", arrays)
    mapped = w.SafeTensors(tmp_path / "f32.safetensors")
    for name, expected in arrays.items():
        np.testing.assert_array_equal(mapped[name], expected)
    bits = (arrays["x"].view(np.uint32) >> 16).astype("<u2")
    header = json.dumps({"x": {"dtype": "BF16", "shape": [3, 7], "data_offsets": [0, bits.nbytes]}}).encode()
    (tmp_path / "bf16.safetensors").write_bytes(struct.pack("<Q", len(header)) + header + bits.tobytes())
    bf16 = w.SafeTensors(tmp_path / "bf16.safetensors")["x"]
    np.testing.assert_array_equal(bf16[1:2], arrays["x"][1:2])
    np.testing.assert_array_equal(np.asarray(bf16), arrays["x"])
    dtype, raw = w.stored_tensor({"x": bf16}, "x")
    assert dtype == w.DTYPE_BF16 and raw.dtype == np.uint16
    np.testing.assert_array_equal(raw, bits)


def test_bf16_writer_rounds_to_nearest_even(pkg, tmp_path):
    w = pkg.weights
    values = np.array([1.0, 1.00390625, 1.01171875, -3.14159, 65504.0, 1e-30], np.float32)
    w.save_safetensors(tmp_path / "b.safetensors", {"v": values}, dtype="BF16")
    got = np.asarray(w.SafeTensors(tmp_path / "b.safetensors")["v"])
    import torch
    expected = torch.from_numpy(values).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(got, expected)


@pytest.mark.parametrize("payload", [b"", struct.pack("<Q", 1024) + b"{}",
                                     struct.pack("<Q", 62) + b'{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}'])
def test_truncated_weights_rejected(pkg, tmp_path, payload):
    path = tmp_path / "bad.safetensors"
    path.write_bytes(payload)
    with pytest.raises((ValueError, KeyError)):
        pkg.weights.SafeTensors(path)


def test_shards_and_path_containment(pkg, tmp_path):
    w = pkg.weights
    w.save_safetensors(tmp_path / "part.safetensors", {"x": np.ones((3,), np.float32)})
    index = tmp_path / "model.safetensors.index.json"
    index.write_text(json.dumps({"weight_map": {"x": "part.safetensors"}}))
    np.testing.assert_array_equal(w.ShardedSafeTensors(index)["x"], np.ones(3))
    index.write_text(json.dumps({"weight_map": {"x": "../outside.safetensors"}}))
    with pytest.raises(ValueError, match="escapes"):
        w.ShardedSafeTensors(index)


def test_config_roundtrip_and_validation(pkg):
    config = cases.micro_config("nano15")
    ModelConfig = pkg.ModelConfig
    assert ModelConfig.from_dict(json.loads(json.dumps(config.to_dict()))) == config
    for changes in ({"head_dim": 3}, {"query_heads": 3}, {"layers": True}, {"window": 0},
                    {"norm_eps": float("nan")}, {"global_layers": (0,)}, {"family": "miracle-neural"}):
        with pytest.raises(ValueError):
            replace(config, **changes)
    with pytest.raises(ValueError, match="scope"):
        ModelConfig.from_dict({"model_type": "miracle_neural"})


def test_native_checkpoint_names_resolve(pkg):
    config = cases.micro_config("heavy_mid")
    weights = cases.micro_weights(config)
    names = pkg.weights.native_names(config)
    native = {names[k]: v for k, v in weights.items()}
    adapted = pkg.weights.adapt_weights(config, native)
    for key in weights:
        np.testing.assert_array_equal(adapted[key], weights[key])


def test_bad_weights_rejected_before_device_allocation(pkg):
    # tests/test_inference.py:102-106: shape errors surface before any device work
    config = cases.micro_config("nano15")
    weights = cases.micro_weights(config)
    weights["layers.0.k"] = np.zeros((7, 16), np.float32)
    with pytest.raises(ValueError, match="expected"):
        submodule("model").MiracleModel(config, weights)


def test_hash_generator_is_deterministic_and_normal_shaped(pkg):
    syn = cases.synthetic
    a = syn.hash_normal_bf16(0, 3, (64, 1024), 0.02)
    b = syn.hash_normal_bf16(0, 3, (64, 1024), 0.02, chunk=1000)
    np.testing.assert_array_equal(a, b)
    values = np.asarray(pkg.weights.BF16Array(a))
    assert abs(values.mean()) < 1e-3 and abs(values.std() - 0.02) < 5e-4
    assert not np.array_equal(a, syn.hash_normal_bf16(0, 4, (64, 1024), 0.02))
    part = syn.hash_normal_f32(0, 3, 5000, 100, 0.02)
    np.testing.assert_array_equal(pkg.weights.float32_to_bf16_bits(part), a.reshape(-1)[5000:5100])


def test_unpinned_choices_are_recorded():
    syn = cases.synthetic
    lighting, heavy = syn.config_for("lighting"), syn.config_for("heavy")
    assert lighting.kv_heads == syn.UNPINNED_CHOICES["lighting"]["kv_heads"]
    assert lighting.memory_slots == 0 and lighting.window == syn.UNPINNED_CHOICES["lighting"]["window"]
    total = sum(int(np.prod(s)) for s in cases.expected_shapes(heavy).values())
    assert 35e9 < total < 40e9


# ---- C ABI: the library loads and exports everything the header declares ----------
def _declared_symbols():
    header = (REPO / "include" / "miracle_cuda.h").read_text()
    return sorted(set(re.findall(r"\bMR_API\s+(?:const\s+char\s*\*|int)\s*(mr_\w+)\s*\(", header)))


def test_header_declarations_are_all_exported():
    lib_path = REPO / "miraclereasoning-cpu_b200" / "libmiracle_cuda.so"
    assert lib_path.exists(), "build libmiracle_cuda.so first (python miraclereasoning-cpu_b200/build.py)"
    lib = ctypes.CDLL(str(lib_path))
    declared = _declared_symbols()
    assert len(declared) >= 40
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    lib.mr_abi_version.restype = ctypes.c_int
    assert lib.mr_abi_version() == 1


def test_python_binding_covers_the_header():
    assert sorted(submodule("_native").SIGNATURES) == _declared_symbols()


def test_engine_config_flattening():
    cfg = submodule("model").engine_config(cases.micro_config("heavy_mid"), 96)
    assert (cfg.family, cfg.routed_experts, cfg.block_size, cfg.global_slots) == (5, 16, 4, 3)
    assert cfg.alibi_slope == pytest.approx(0.015 / 4)
    assert ctypes.sizeof(cfg) == 30 * 4  # 30 four-byte fields of mr_model_config, no padding


# ---- which device path runs a family, and the decisions it reports ------------------
def test_engine_plans_routes_families():
    model = importlib.import_module("miraclereasoning-cpu_b200.model")
    for name in ("nano15", "nano17", "lite", "lighting", "heavy"):
        assert model.engine_plans(cases.synthetic.config_for(name)), name
    assert model.engine_plans(cases.micro_config("nano16"))         # chunk relays pooled between steps
    assert model.engine_plans(cases.micro_config("lighting"))       # memory slots merged between steps
    assert model.engine_plans(cases.micro_config("lighting_drop"))
    # FlashLighting's latent mask needs a window (the reference fails without one)
    windowless = dataclasses.replace(cases.micro_config("lighting_drop"), window=None)
    assert not model.engine_plans(windowless)


def test_ring_decisions_follow_the_drop_path():
    """FlashLighting without memory slots keeps positions max(0, p + 1 - window) .. p."""
    model = importlib.import_module("miraclereasoning-cpu_b200.model")
    config = cases.micro_config("lighting_drop")

    class Stub:
        pass

    stub = Stub()
    stub.config, stub.position = config, 7
    decisions = model.RingDecisions(stub)
    assert len(decisions) == 7
    assert decisions[0] == [{"latent_positions": [[0]], "memory_size": [0]}] * config.layers
    w = config.window
    assert decisions[6][0]["latent_positions"] == [list(range(7 - w, 7))]
    with pytest.raises(IndexError):
        decisions[7]


def test_bench_heavy_byte_accounting():
    """Heavy Medium reads its layer weights once per inner loop and only the chosen experts."""
    bench = importlib.import_module("bench")
    config = cases.micro_config("heavy_mid")
    shapes = cases.expected_shapes(config)
    expert = sum(int(np.prod(shapes[f"layers.0.experts.0.{k}"])) * 4 for k in ("gate", "up", "down"))
    base = bench.weight_bytes(config, "F32", 0)
    assert bench.weight_bytes(config, "F32", 2) - base == 2 * expert * config.layers * config.inner_loop_steps
    assert bench.launches_per_step(config) == 1 + 6 * config.layers * config.inner_loop_steps + 2
    assert bench.launches_per_step(config, True) == 1 + 8 * config.layers * config.inner_loop_steps + 2
    assert bench.launches_per_step(cases.micro_config("nano15")) == 1
