"""The allocation-free dispatch plan (smoe_dispatch_plan_noalloc).

It exists for callers that cannot allocate device memory -- a host that owns all device
memory in its own arena or caching allocator and must not have a library call cudaMalloc
behind its back (which would also synchronise the device mid-step).  The test drives it
through the C ABI and checks it against the regular workspace-taking entry point,
smoe_dispatch_plan, on two calls in a row with different sizes, so that the second call
runs on scratch left behind by the first.  Collected last (file name) so that a run that
stops at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _routing(T, k, E, seed):
    rng = np.random.default_rng(seed)
    p = rng.dirichlet(np.ones(E) * 0.5) + 1e-3
    p /= p.sum()
    idx = np.array([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)], dtype=np.int32)
    return torch.from_numpy(idx.reshape(T, k)).cuda()


def _noalloc_plan(lib, idx, E, capacity, row_align):
    from swiftmoe_b200 import _lib as L
    T, k = idx.shape
    rows_cap = int(lib.smoe_plan_rows_cap(T, k, E, capacity, row_align))
    dev = idx.device
    out = dict(counts=torch.full((E,), -7, dtype=torch.int32, device=dev),
               offsets=torch.full((E + 1,), -7, dtype=torch.int32, device=dev),
               slot_row=torch.full((T * k,), -7, dtype=torch.int32, device=dev),
               row_token=torch.full((max(rows_cap, 1),), -7, dtype=torch.int32, device=dev))
    rc = lib.smoe_dispatch_plan_noalloc(idx.data_ptr(), T, k, E, capacity, row_align, out["counts"].data_ptr(),
                                        out["offsets"].data_ptr(), out["slot_row"].data_ptr(),
                                        out["row_token"].data_ptr(), max(rows_cap, 1), L.stream_handle(dev))
    L.check(rc, "smoe_dispatch_plan_noalloc")
    return out


def test_noalloc_plan_matches_workspace_plan():
    from swiftmoe_b200 import _lib as L
    from swiftmoe_b200 import kernels
    lib = L.load()
    cases = [(20000, 8, 128, 900, 8), (3000, 2, 64, 100, 1)]   # two calls in a row, different sizes
    for (T, k, E, cap, align) in cases:
        idx = _routing(T, k, E, seed=T)
        ref = kernels.dispatch_plan(idx, E, cap, align)
        got = _noalloc_plan(lib, idx, E, cap, align)
        torch.cuda.synchronize()
        assert torch.equal(got["counts"], ref["counts"])
        assert torch.equal(got["offsets"], ref["offsets"])
        assert torch.equal(got["slot_row"], ref["slot_row"])
        total = int(ref["offsets"][-1])
        assert torch.equal(got["row_token"][:total], ref["row_token"][:total])


def test_noalloc_plan_rejects_sizes_beyond_its_scratch():
    from swiftmoe_b200 import _lib as L
    lib = L.load()
    max_slots, max_e = 1 << 19, 256
    # nothing is dereferenced or launched: the size check comes first
    assert lib.smoe_dispatch_plan_noalloc(None, max_slots // 2 + 1, 2, 8, 0, 1, None, None, None, None,
                                          max_slots + 2, None) == -6
    assert lib.smoe_dispatch_plan_noalloc(None, 10, 2, max_e + 1, 0, 1, None, None, None, None, 20, None) == -6
    assert L.load().smoe_status_string(-6).decode().startswith("size beyond")
