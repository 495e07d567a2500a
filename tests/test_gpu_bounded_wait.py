"""The give-up path of the library's bounded device waits, exercised without a hang:
a self-test kernel waits on an mbarrier that nothing arrives at with a 1 ms limit, the
wait returns, the timeout is reported through the device error word, and the context
keeps working (a grouped GEMM right after it computes correct results and leaves the
error word at zero)."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_gives_up_and_reports_timeout():
    from swiftmoe_b200 import _lib as L, kernels as K
    lib = L.load()
    dev = torch.device("cuda", 0)
    K.read_device_error(dev)                         # start from a clear error word
    gave_up = torch.zeros(1, dtype=torch.int32, device=dev)
    L.check(lib.smoe_selftest_wait_timeout(1_000_000, L.ptr(gave_up), L.stream_handle(dev)),
            "smoe_selftest_wait_timeout")
    torch.cuda.synchronize()
    assert int(gave_up.item()) == 1
    assert K.read_device_error(dev) == 1             # kErrWaitTimeout, and the read clears it
    assert K.read_device_error(dev) == 0
    # the context is intact: an ordinary tensor-core GEMM afterwards is correct
    g = torch.Generator(device=dev).manual_seed(3)
    A = torch.randn(300, 256, device=dev, generator=g).to(torch.bfloat16)
    B = torch.randn(2, 512, 256, device=dev, generator=g).to(torch.bfloat16)
    offs = torch.tensor([0, 120, 300], dtype=torch.int32, device=dev)
    C_ = K.grouped_gemm(A, B, offs)
    ref = torch.cat([A[:120].float() @ B[0].float().T, A[120:].float() @ B[1].float().T])
    err = (C_.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2
    assert K.read_device_error(dev) == 0
