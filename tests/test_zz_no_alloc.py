"""The allocation-free attention entry point (mr_attention_static_scratch).

Some callers cannot call cudaMalloc while they run: a framework that owns all
device memory through its own pool, or code in a section where an allocation
could synchronise the device or fail under memory pressure.  For them the
library offers attention whose score matrix lives in a fixed 4 MiB device
array instead of a per-call buffer.  This test calls that entry point through
the C ABI on device memory the test owns (torch tensors) and checks it against
the regular, allocating path (CUDABackend.attention = mr_op_scores +
mr_op_softmax + mr_op_mix) within the kernel-test tolerance (and bit for bit),
on several calls in a row with different shapes (each call reuses the array
the one before it left behind): a ring with extra rows, a ring alone, a start
near INT_MAX, and extra rows with no ring.  It also checks that an oversize
request is refused.

It sits in its own file named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import submodule

pytestmark = pytest.mark.gpu


def _device(array):
    import torch
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).cuda()


def test_static_scratch_attention_matches_the_allocating_path(backend):
    import torch
    native = submodule("_native")
    lib = native.library()
    shapes = [  # heads, kv_heads, dim, capacity, start, length, extra_length
        (8, 2, 32, 64, 50, 40, 6),
        (16, 4, 64, 300, 290, 256, 0),
        # a start near INT_MAX: ring rows are (start + t) mod capacity in 64-bit arithmetic
        (8, 2, 32, 300, 2**31 - 7, 200, 3),
        # only extra rows: no ring at all (NULL keys/values, capacity 0)
        (4, 1, 16, 0, 0, 0, 9),
    ]
    for call, (heads, kvh, dim, cap, start, length, extra) in enumerate(shapes):
        rng = np.random.default_rng(100 + call)
        q = rng.normal(size=(1, heads * dim)).astype(np.float32)
        keys, values = (rng.normal(size=(max(cap, 1), kvh * dim)).astype(np.float32) for _ in range(2))
        ek, ev = (rng.normal(size=(max(extra, 1), kvh * dim)).astype(np.float32) for _ in range(2))
        b = backend
        ring_k, ring_v = (b.upload(keys), b.upload(values)) if length else (b.upload(ek), b.upload(ev))
        want = b.read(b.attention(b.upload(q), ring_k, ring_v, heads=heads, kv_heads=kvh, dim=dim,
                                  start=start, length=length,
                                  extra_keys=b.upload(ek) if extra else None,
                                  extra_values=b.upload(ev) if extra else None, extra_length=extra))
        tq, tk, tv, tek, tev = (_device(a) for a in (q, keys, values, ek, ev))
        out = torch.full((heads * dim,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        rc = lib.mr_attention_static_scratch(backend.context, tq.data_ptr(),
                                             tk.data_ptr() if length else None, tv.data_ptr() if length else None,
                                             tek.data_ptr(), tev.data_ptr(), out.data_ptr(), heads, kvh, dim, cap,
                                             start, length, extra)
        assert rc == 0, lib.mr_last_error().decode()
        native.call("mr_context_finish", backend.context)
        got = out.cpu().numpy()
        np.testing.assert_allclose(got, want.reshape(-1), rtol=1e-6, atol=1e-6)
        # same dot products, the softmax sum in row order, the mix in row order: bit for bit
        np.testing.assert_array_equal(got, want.reshape(-1))


def test_static_scratch_attention_refuses_oversize_requests(backend):
    import torch
    native = submodule("_native")
    lib = native.library()
    t = torch.zeros(64, device="cuda")
    # 64 heads x 20000 rows = 1,280,000 scores > the 1,048,576-float array
    rc = lib.mr_attention_static_scratch(backend.context, t.data_ptr(), t.data_ptr(), t.data_ptr(), None, None,
                                         t.data_ptr(), 64, 1, 1, 20000, 0, 20000, 0)
    assert rc == native.MR_ERR_ARGUMENT
    assert "static scratch holds" in lib.mr_last_error().decode()
