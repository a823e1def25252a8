"""Op-level parity on the GPU: CUDABackend against the reference kernels.

The reference's own kernel tests (tests/test_opencl.py:19-63: same shapes,
seeds and tolerances) run unchanged on the CUDA backend, then every kernel is
compared on random inputs with the CPU oracle (oracle/kernels.c, pinned bit for
bit to kernels.cl).  Sums and products are rounded in the reference order
(FP_CONTRACT OFF), so results agree to the last bit except where CUDA's
exp/sin/cos differ from the host libm by an ulp: tolerance 1e-6 relative.
"""
import numpy as np
import pytest

import cases
from oracle.host_backend import HostBackend, SIGNATURES
from test_oracle import _random_args

pytestmark = pytest.mark.gpu


def test_primitives_with_non_aligned_shapes(backend):
    b = backend
    rng = np.random.default_rng(9)
    x = rng.normal(size=(3, 19)).astype(np.float32)
    w = rng.normal(size=(7, 19)).astype(np.float32)
    np.testing.assert_allclose(b.read(b.linear(b.upload(x), b.upload(w))), x @ w.T, atol=4e-6)
    scales = rng.normal(size=19).astype(np.float32)
    expected = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + 1e-6) * scales
    np.testing.assert_allclose(b.read(b.norm(b.upload(x), b.upload(scales), 19, 1e-6)), expected, atol=1e-6)
    logits = np.array([[1000, 1001, -1000], [-1000, -1001, -1002]], np.float32)
    e = np.exp(logits - logits.max(axis=1, keepdims=True))
    np.testing.assert_allclose(b.read(b.softmax(b.upload(logits))), e / e.sum(axis=1, keepdims=True), atol=1e-7)


@pytest.mark.parametrize("split", [False, True])
def test_rope_layouts(backend, split):
    rng = np.random.default_rng(3)
    x = rng.normal(size=(2, 3, 6)).astype(np.float32)
    pos = np.array([7, 29], np.float32)
    freq = np.array([1, .1, .01], np.float32)
    angles = pos[:, None, None] * freq[None, None, :]
    first, second = (x[..., :3], x[..., 3:]) if split else (x[..., ::2], x[..., 1::2])
    u, v = first * np.cos(angles) - second * np.sin(angles), first * np.sin(angles) + second * np.cos(angles)
    expected = np.concatenate([u, v], axis=-1) if split else np.stack([u, v], axis=-1).reshape(2, 3, 6)
    actual = backend.rotate(backend.upload(x.reshape(2, 18)), backend.upload(freq), backend.upload(pos), 3, 6, split)
    np.testing.assert_allclose(backend.read(actual).reshape(x.shape), expected, atol=3e-6)


def test_attention_group_mapping_ring_and_relays(backend):
    b, rng = backend, np.random.default_rng(6)
    q = rng.normal(size=(4, 6)).astype(np.float32)
    k, v = [rng.normal(size=(5, 2, 6)).astype(np.float32) for _ in range(2)]
    rk, rv = [rng.normal(size=(3, 2, 6)).astype(np.float32) for _ in range(2)]
    keys, values = np.concatenate([k[[3, 4, 0, 1]], rk]), np.concatenate([v[[3, 4, 0, 1]], rv])
    expected = []
    for head in range(4):
        logits = keys[:, head // 2] @ q[head] / np.sqrt(6)
        probs = np.exp(logits - logits.max())
        probs /= probs.sum()
        expected.append(probs @ values[:, head // 2])
    actual = b.attention(b.upload(q.reshape(1, -1)), b.upload(k.reshape(5, -1)), b.upload(v.reshape(5, -1)),
                         heads=4, kv_heads=2, dim=6, start=3, length=4,
                         extra_keys=b.upload(rk.reshape(3, -1)), extra_values=b.upload(rv.reshape(3, -1)),
                         extra_length=3)
    np.testing.assert_allclose(b.read(actual).reshape(4, 6), expected, atol=1e-6)


def test_known_answer_fixtures(backend):
    g = np.load(cases.GOLDEN_DIR / "kernels.npz")
    b = backend
    np.testing.assert_array_equal(b.read(b.linear(b.upload(g["lin_x"]), b.upload(g["lin_w"]))), g["lin_y"])
    np.testing.assert_allclose(b.read(b.norm(b.upload(g["lin_x"]), b.upload(g["rms_w"]), 19, 1e-6)), g["rms_y"],
                               rtol=1e-6, atol=0)
    np.testing.assert_allclose(b.read(b.softmax(b.upload(g["sm_x"]))), g["sm_y"], rtol=1e-6, atol=1e-30)


@pytest.mark.parametrize("name", sorted(SIGNATURES))
def test_every_kernel_matches_oracle(backend, name):
    host = HostBackend("oracle")
    for seed in range(3):
        shape, args = _random_args(name, np.random.default_rng(seed))
        outs = {}
        for label, b in (("gpu", backend), ("cpu", host)):
            tensors, call_args = [], []
            for a in args:
                if isinstance(a, np.ndarray):
                    t = b.upload(a)
                    tensors.append(t)
                    call_args.append(t)
                else:
                    call_args.append(a)
            b.run(name, shape, *call_args)
            outs[label] = [b.read(t) for t in tensors]
        for g, c in zip(outs["gpu"], outs["cpu"]):
            np.testing.assert_allclose(g, c, rtol=1e-6, atol=1e-6)


def test_out_of_bounds_arguments_raise_before_launch(backend, pkg):
    b = backend
    x, w = b.upload(np.ones((2, 4), np.float32)), b.upload(np.ones((3, 4), np.float32))
    out = b.empty((2, 3))
    with pytest.raises(pkg.CUDAError, match="needs"):
        b.run("linear", (3, 2), x, w, out, 2, 3, 8)   # in_dim larger than the buffers
    with pytest.raises(ValueError, match="out of bounds"):
        b.copy(x, out, source_offset=5, count=4)
