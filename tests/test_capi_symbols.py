"""The C-ABI library loads without a GPU and exports every symbol include/swiftmoe.h
declares; host-only entry points answer without touching a device."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "swiftmoe.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"SMOE_API\s+[\w\s\*]+?\b(smoe_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from swiftmoe_b200 import build, _lib
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n


def test_bindings_cover_header(lib):
    from swiftmoe_b200 import _lib
    assert set(declared()) == set(_lib.SIGNATURES)


def test_host_only_queries(lib):
    assert lib.smoe_version().decode().startswith("swiftmoe-b200")
    assert lib.smoe_status_string(-1).decode() == "invalid argument"
    assert lib.smoe_plan_rows_cap(100, 2, 8, 0, 1) == 200
    assert lib.smoe_plan_rows_cap(100, 2, 8, 10, 1) == 80
    assert lib.smoe_plan_rows_cap(100, 2, 8, 0, 128) == 200 + 8 * 127
    assert lib.smoe_plan_workspace_size(100, 2, 8) > 0
    assert lib.smoe_router_workspace_size(16384, 4096, 8, 2) == 0          # fused small-E path
    assert lib.smoe_router_workspace_size(16384, 2048, 128, 2) >= 16384 * 128 * 4
    assert lib.smoe_ep_regroup_workspace_size(8, 1) > 0


def test_invalid_arguments_rejected_before_any_device_call(lib):
    from swiftmoe_b200 import _lib
    # k > E, k > 32, bad dtype: rejected by validation, no CUDA call is made
    assert lib.smoe_router_fwd(None, None, 2, None, 10, 64, 4, 5, None, None, None, None, 0, None) == -1
    assert lib.smoe_topk_from_logits(None, 10, 64, 33, None, None, None) == -1
    assert lib.smoe_grouped_gemm(None, None, None, None, 2, 2, 0, None, None, 1, 10, 8, 8, None) == -1
    assert lib.smoe_combine(None, 9, None, None, 1, 2, 8, None, None, None) == -1
    assert lib.smoe_selftest_wait_timeout(0, None, None) == -1               # no limit
    assert lib.smoe_selftest_wait_timeout(2_000_000_000, None, None) == -1   # above 1 s
    a = _lib.LayerArgs()
    a.tokens, a.d_model, a.num_experts, a.top_k, a.dtype = 10, 64, 8, 9, 2
    assert lib.smoe_layer_fwd(C.byref(a), None) == -1
    assert lib.smoe_layer_workspace_size(C.byref(a)) > 0
