"""Host-side logic of the drop-in modules (no GPU): constructor/attribute/parameter
parity with the reference, capacity arithmetic, and the no-CPU-fallback rule."""
import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import swiftmoe_b200 as S
from swiftmoe_b200._core import capacity_rows, resolve_dtype
from swiftmoe_b200._lib import SwiftMoEError


def test_ultimate_defaults_and_params():
    m = S.UltimateMoE(num_experts=8, d_model=32)
    assert (m.num_experts, m.d_model, m.exp_per_rank, m.ws, m.rank) == (8, 32, 8, 1, 0)
    assert m.use_fp16 and m.use_triton and m.use_nccl_opt and not m.enable_profiling
    assert m.expert_weights.shape == (8, 32, 32) and m.expert_weights.dtype == torch.float16
    assert m.gate_weight.shape == (8, 32)
    assert set(dict(m.named_parameters())) == {"expert_weights", "gate_weight"}
    s = m.get_profile_summary()
    assert set(s) >= {"Router", "Dispatch_Comm", "Expert_Compute", "Combine_Comm"}


def test_standard_params_match_reference_names():
    m = S.StandardMoE(num_experts=8, d_model=16, use_fp16=False)
    names = set(dict(m.named_parameters()))
    assert names == {"gate.weight"} | {f"experts.{i}.weight" for i in range(8)}
    assert m.experts_per_rank == 8 and m.world_size == 1
    assert S.BaselineMoE is S.StandardMoE
    for meth in ("_route_tokens", "_dispatch_tokens", "_expert_forward", "_combine_tokens"):
        assert callable(getattr(m, meth))


def test_reference_state_dict_loads(golden_dir):
    """A state_dict of the reference StandardMoE loads unchanged (same names/layouts)."""
    ref_sd = {"gate.weight": torch.randn(8, 16)}
    ref_sd.update({f"experts.{i}.weight": torch.randn(16, 16) for i in range(8)})
    m = S.StandardMoE(num_experts=8, d_model=16, use_fp16=False)
    m.load_state_dict(ref_sd)
    assert torch.equal(m.experts[3].weight, ref_sd["experts.3.weight"])
    u = S.UltimateMoE(num_experts=8, d_model=16, use_fp16=False)
    u.load_state_dict({"gate_weight": torch.randn(8, 16), "expert_weights": torch.randn(8, 16, 16)})


def test_swiglu_extension_shapes():
    m = S.UltimateMoE(8, 32, use_fp16=False, dtype="bf16", top_k=2, expert_type="swiglu", d_ff=48,
                      num_shared_experts=1, d_ff_shared=24)
    assert m.w1.shape == (8, 48, 32) and m.w3.shape == (8, 48, 32) and m.w2.shape == (8, 32, 48)
    assert m.shared_w1.shape == (24, 32) and m.shared_w2.shape == (32, 24)
    assert m.compute_dtype == torch.bfloat16


def test_no_cpu_fallback():
    m = S.UltimateMoE(8, 32, use_fp16=False)
    with pytest.raises(SwiftMoEError):
        m(torch.randn(4, 32))
    with pytest.raises(ValueError):
        m(torch.randn(4, 31))


def test_invalid_configs():
    with pytest.raises(ValueError):
        S.UltimateMoE(8, 32, top_k=9)
    with pytest.raises(ValueError):
        S.UltimateMoE(8, 32, expert_type="gelu")
    with pytest.raises(ValueError):
        S.StandardMoE(8, 32, world_size=2)   # no process group of size 2


def test_capacity_and_dtype_helpers():
    assert capacity_rows(None, 100, 1, 2, 8) == 0
    # C3: cf 1.25, 8192 tokens/GPU on 8 GPUs, 64 experts, top-2 -> 2560 rows per expert
    assert capacity_rows(1.25, 8192, 8, 2, 64) == 2560
    assert capacity_rows(1.25, 10, 1, 2, 8) == math.ceil(1.25 * 10 * 2 / 8)
    assert resolve_dtype(True, None) == torch.float16
    assert resolve_dtype(False, None) == torch.float32
    assert resolve_dtype(True, "bf16") == torch.bfloat16


def test_setup_nccl_optimizations_does_not_override(monkeypatch):
    monkeypatch.setenv("NCCL_P2P_LEVEL", "SYS")
    cfg = S.setup_nccl_optimizations()
    import os
    assert os.environ["NCCL_P2P_LEVEL"] == "SYS"
    assert "NCCL_P2P_LEVEL" in cfg


def test_product_does_not_import_oracle():
    """The checker (oracle/) is never imported by the product package."""
    from pathlib import Path
    import swiftmoe_b200
    for p in Path(swiftmoe_b200.__file__).parent.glob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p


REFERENCE_RECORD_KEYS = {  # experiments/benchmark_suite.py:134-152
    "model_type", "world_size", "batch_size", "num_experts", "d_model", "use_triton", "use_nccl_opt",
    "latency_mean_ms", "latency_std_ms", "latency_min_ms", "latency_max_ms", "latency_p50_ms",
    "latency_p95_ms", "latency_p99_ms", "throughput_tokens_per_sec", "max_memory_gb"}


def test_bench_records_grid_matches_reference():
    from swiftmoe_b200.bench_records import reference_grid
    grid = reference_grid()
    assert {e for e, _ in grid} == {64, 128, 256}
    assert {b for _, b in grid} == {512, 1024, 2048, 4096, 8192}


def test_chunk_bounds_same_count_for_every_batch_size():
    """The chunked schedules exchange one count vector per chunk, so the chunk count may
    not depend on the rank's batch size (ranks may hold different numbers of tokens)."""
    from swiftmoe_b200.ep import chunk_bounds
    for T in (0, 1, 3, 4, 23, 1000):
        b = chunk_bounds(T, 4)
        assert len(b) == 4
        assert b[0][0] == 0 and b[-1][1] == T
        assert all(b[i][1] == b[i + 1][0] and b[i][0] <= b[i][1] for i in range(3))


def test_kept_rows_and_capacity_positions():
    from swiftmoe_b200.ep import capacity_positions, kept_rows
    assert kept_rows(np.array([5, 0, 9]), 0) == 14
    assert kept_rows(np.array([5, 0, 9]), 4) == 8
    rc = np.array([[[2, 0], [1, 3]], [[4, 1], [0, 2]]])            # [chunk, src, expert]
    pos = capacity_positions(rc, 3)
    # source-major, then chunk: src 0 chunk 0, src 0 chunk 1, src 1 chunk 0, src 1 chunk 1
    assert pos[:, 0, 0].tolist() == [0, 2] and pos[:, 1, 0].tolist() == [6, 7]
    assert pos[:, 0, 1].tolist() == [0, 0] and pos[:, 1, 1].tolist() == [1, 4]


def test_bench_host_helpers(monkeypatch):
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import bench
    assert bench._cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert bench._cpulist("") == set()
    # without a GPU the topology is unknown: no binding, no exception
    assert bench.bind_near_gpu(0) is None
    for name, wl in bench.WORKLOADS.items():
        assert {"d", "E", "k", "F", "T", "dtype", "cf", "shared", "bias_std", "name"} <= set(wl), name
        assert wl["E"] % 8 == 0, name          # expert parallelism up to 8 GPUs
