"""Whole-layer parity of the drop-in modules: reference fixtures (fp32, max-abs 1e-5)
and the oracle on rounded inputs (bf16 / fp16, max-rel 2e-2)."""
import numpy as np
import pytest
import torch

import fixtures as fx
import synth
from oracle import moe_oracle as O
from util import max_abs_err, max_rel_err, rounded, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def M():
    import swiftmoe_b200
    return swiftmoe_b200


def _std_from_params(M, p, E, d, dtype, **kw):
    m = M.StandardMoE(E, d, use_fp16=False, dtype=dtype, **kw).cuda()
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy(p.gate))
        if p.expert_type == "linear":
            for i in range(E):
                m.experts[i].weight.copy_(torch.from_numpy(p.expert_w[i].T.copy()))
        else:
            for i in range(E):
                m.experts[i].w1.weight.copy_(torch.from_numpy(p.w1[i]))
                m.experts[i].w3.weight.copy_(torch.from_numpy(p.w3[i]))
                m.experts[i].w2.weight.copy_(torch.from_numpy(p.w2[i]))
    return m


@pytest.mark.parametrize("name", fx.STD_LINEAR)
def test_standard_linear_fp32_vs_reference(M, name):
    f, p = fx.std_linear(name)
    m = _std_from_params(M, p, f["E"], f["d"], torch.float32)
    out = m(to_dev(f["x"])).cpu().numpy()
    assert out.shape == f["out"].shape
    assert max_abs_err(out, f["out"]) <= 1e-5


@pytest.mark.parametrize("name", fx.STD_SWIGLU)
def test_standard_swiglu_fp32_vs_reference(M, name):
    f, p = fx.std_swiglu(name)
    m = _std_from_params(M, p, f["E"], f["d"], torch.float32, expert_type="swiglu", d_ff=f["F"])
    out = m(to_dev(f["x"])).cpu().numpy()
    assert max_abs_err(out, f["out"]) <= 1e-5


def test_ultimate_linear_fp32_vs_reference_ws1(M):
    f, p = fx.ult_linear("ult_linear_fp32_ws1_E8_d64_M50")
    m = M.UltimateMoE(f["E"], f["d"], use_fp16=False).cuda()
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(p.gate))
        m.expert_weights.copy_(torch.from_numpy(p.expert_w))
    out = m(to_dev(f["x"][0])).cpu().numpy()
    assert max_abs_err(out, f["out"][0]) <= 1e-5


def test_standard_linear_fp16_vs_reference(M):
    f, p = fx.std_linear("std_linear_fp16_E8_d128_M33")
    m = _std_from_params(M, p, f["E"], f["d"], torch.float16)
    out = m(to_dev(f["x"], torch.float16)).float().cpu().numpy()
    ref = f["out"]
    assert np.abs(out - ref).max() <= 2e-3 * np.abs(ref).max()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,d,E,k,F,cf,shared,bias", [
    (1, 256, 8, 2, 512, None, False, False),
    (1, 256, 8, 1, 512, None, True, True),       # decode: rows gathered by the gate/up kernel
    (2, 512, 16, 1, 256, 1.0, True, True),
    (257, 512, 8, 2, 1024, None, False, False),
    (1000, 256, 64, 2, 256, 1.25, False, False),
    (600, 256, 32, 8, 128, None, True, True),
    (2048, 512, 128, 8, 128, 1.25, True, True),
])
def test_swiglu_layer_vs_oracle(M, dtype, T, d, E, k, F, cf, shared, bias):
    rng_seed = T + E
    w1, w3, w2 = synth.swiglu_weights(rng_seed, E, d, F, init="normal", std=0.02)
    g = synth.normal(rng_seed + 5, (E, d), 0.02)
    x = synth.normal(rng_seed + 9, (T, d), 1.0)
    lb = synth.normal(rng_seed + 2, (E,), 1.5) if bias else None
    sw = synth.swiglu_weights(rng_seed + 1, 1, d, F, init="normal", std=0.02) if shared else None
    r = lambda a: rounded(a, dtype)
    m = M.UltimateMoE(E, d, use_fp16=False, dtype=dtype, top_k=k, expert_type="swiglu", d_ff=F,
                      capacity_factor=cf, num_shared_experts=1 if shared else 0, d_ff_shared=F).cuda()
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(g))
        m.w1.copy_(torch.from_numpy(w1)); m.w3.copy_(torch.from_numpy(w3)); m.w2.copy_(torch.from_numpy(w2))
        if shared:
            m.shared_w1.copy_(torch.from_numpy(sw[0][0])); m.shared_w3.copy_(torch.from_numpy(sw[1][0]))
            m.shared_w2.copy_(torch.from_numpy(sw[2][0]))
    if bias:
        m.set_logit_bias(torch.from_numpy(lb))
    out = m(to_dev(x, dtype)).float().cpu().numpy()
    p = O.MoEParams(gate=r(g), expert_type="swiglu", w1=r(w1), w3=r(w3), w2=r(w2), logit_bias=lb)
    if shared:
        p.sw1, p.sw3, p.sw2 = r(sw[0]), r(sw[1]), r(sw[2])
    # fp32 (here float64) oracle on the same rounded inputs and weights
    (ref,), aux = O.moe_forward([r(x)], p, k=k, capacity_factor=cf, acc=np.float64, return_aux=True)
    # routing may only differ on near-ties; compare rows whose routing agrees exactly
    idx, _ = __import__("swiftmoe_b200").kernels.router(to_dev(x, dtype), m.gate_weight, k,
                                                        m.logit_bias)
    same = (idx.cpu().numpy() == aux["routed"][0][0]).all(1)
    assert same.mean() > 0.99
    rows = same if cf is None else np.arange(T) < (np.argmin(same) if not same.all() else T)
    # (with a capacity a routing flip can move the cut for later tokens: compare the rows
    # before the first flip)
    assert max_rel_err(out[rows], ref[rows]) <= 2e-2
    nrm = np.linalg.norm(out[rows] - ref[rows]) / max(np.linalg.norm(ref[rows]), 1e-30)
    assert nrm <= 1e-2


def test_layer_empty_and_single(M):
    m = M.UltimateMoE(8, 64, use_fp16=False, dtype=torch.bfloat16, expert_type="swiglu", d_ff=128).cuda()
    assert m(torch.empty((0, 64), device="cuda", dtype=torch.bfloat16)).shape == (0, 64)
    assert m(torch.randn((1, 64), device="cuda", dtype=torch.bfloat16)).shape == (1, 64)


def test_fp16_default_reference_smoke_shape(M):
    """scripts/test_setup.py:545-575: StandardMoE(8,128) / UltimateMoE(8,128), 32 tokens fp16."""
    for m in (M.StandardMoE(num_experts=8, d_model=128, use_fp16=True),
              M.UltimateMoE(num_experts=8, d_model=128, use_fp16=True, use_triton=False)):
        m = m.cuda()
        x = torch.randn(32, 128, device="cuda", dtype=torch.float16)
        with torch.no_grad():
            assert m(x).shape == x.shape


def test_profiling_summary(M):
    m = M.UltimateMoE(8, 256, use_fp16=False, dtype=torch.bfloat16, expert_type="swiglu", d_ff=512,
                      enable_profiling=True).cuda()
    x = torch.randn(300, 256, device="cuda", dtype=torch.bfloat16)
    ref = None
    for _ in range(3):
        out = m(x)
    s = m.get_profile_summary()
    assert set(s) >= {"Router", "Dispatch_Comm", "Expert_Compute", "Combine_Comm", "Exposed_A2A"}
    assert all(v >= 0 for v in s.values()) and s["Expert_Compute"] > 0
    m.reset_profiling()
    assert m.get_profile_summary()["Router"] == 0
    m.enable_profiling = False
    torch.testing.assert_close(m(x), out, rtol=0, atol=0)
    m._force_staged = True
    torch.testing.assert_close(m(x), out, rtol=0, atol=0)   # staged == fused, bit for bit


def _reference_chain(m, x):
    """The stage calls of the reference's StandardMoE.forward (models/baseline_moe.py:191-213),
    in its order and with its argument passing, over this library's module."""
    indices, weights = m._route_tokens(x)
    recv_x, recv_idx, recv_weights, send_list, recv_list, rev_idx = m._dispatch_tokens(x, indices, weights)
    expert_output = m._expert_forward(recv_x, recv_idx, recv_weights)
    return m._combine_tokens(expert_output, send_list, recv_list, rev_idx, x.shape[0])


@pytest.mark.parametrize("dtype,kw", [
    (torch.bfloat16, {}), (torch.float32, {}),
    (torch.bfloat16, dict(expert_type="swiglu", d_ff=256)),
    (torch.bfloat16, dict(expert_type="swiglu", d_ff=256, capacity_factor=0.6, num_shared_experts=1)),
    (torch.float16, dict(top_k=3))])
def test_reference_stage_chain_matches_forward(M, dtype, kw):
    """StandardMoE's private stages chained as the reference's forward chains them give
    forward's output bit for bit (the weights travel through _dispatch_tokens' third
    return value into _expert_forward, as in the reference)."""
    m = M.StandardMoE(8, 128, use_fp16=False, dtype=dtype, **kw).cuda()
    x = torch.randn(77, 128, device="cuda", dtype=dtype)
    idx, w = m._route_tokens(x)
    assert idx.dtype == torch.int64 and w.dtype == torch.float32
    recv_x, recv_idx, recv_w, s_list, r_list, _ = m._dispatch_tokens(x, idx, w)
    assert recv_x.shape[0] == recv_idx.shape[0] == recv_w.shape[0] == s_list[0] == r_list[0]
    assert recv_w.shape[1] == 1 and int(recv_idx.min()) >= 0 and int(recv_idx.max()) < 8
    torch.testing.assert_close(_reference_chain(m, x), m(x), rtol=0, atol=0)


def test_expert_stage_accepts_any_row_order(M):
    """_expert_forward groups the rows itself: permuting its input rows permutes its output."""
    m = M.StandardMoE(8, 128, use_fp16=False, dtype=torch.bfloat16, expert_type="swiglu", d_ff=256).cuda()
    x = torch.randn(50, 128, device="cuda", dtype=torch.bfloat16)
    idx, w = m._route_tokens(x)
    rx, ri, rw, *_ = m._dispatch_tokens(x, idx, w)
    perm = torch.randperm(rx.shape[0], device="cuda")
    y = m._expert_forward(rx, ri, rw)
    yp = m._expert_forward(rx[perm].contiguous(), ri[perm], rw[perm])
    torch.testing.assert_close(yp, y[perm], rtol=0, atol=0)


def test_ultimate_reference_chain_with_comm_handler(M):
    """UltimateMoE's forward stages (models/ultimate_moe.py:301-338): the reference's
    MoEAsyncCommHandler constructor and dispatch / combine signatures around
    _expert_compute reproduce forward bit for bit; profile_data has the reference's keys."""
    m = M.UltimateMoE(8, 128, use_fp16=False, dtype=torch.bfloat16, enable_profiling=True).cuda()
    x = torch.randn(64, 128, device="cuda", dtype=torch.bfloat16)
    comm = M.MoEAsyncCommHandler(8, 1, 128, "cuda:0")
    from swiftmoe_b200 import kernels
    idx32, w32 = kernels.router(x, m.gate_weight, 2)
    target_ranks, local_idx = idx32 // m.exp_per_rank, idx32 % m.exp_per_rank
    recv_x, recv_idx, recv_w, s_list, r_list, rev = comm.dispatch(x, idx32, w32, target_ranks.view(-1),
                                                                  local_idx.view(-1))
    expert_out = m._expert_compute(recv_x, recv_idx, recv_w)
    out = comm.combine(expert_out, s_list, r_list, rev, x.shape[0])
    torch.testing.assert_close(out, m(x), rtol=0, atol=0)
    assert set(m.profile_data) >= {"router", "dispatch", "compute", "combine"}
    assert len(m.profile_data["router"]) == 1
    m.reset_profiling()
    assert all(len(v) == 0 for v in m.profile_data.values())


def test_bf16_layer_vs_reference_bf16_output(M):
    """Our bf16 layer against the reference's OWN bf16 forward on identical inputs."""
    f, p = fx.std_swiglu_lowp("std_swiglu_bf16_E8_d512_F1024_M64")
    m = _std_from_params(M, p, f["E"], f["d"], torch.bfloat16, expert_type="swiglu", d_ff=f["F"])
    out = m(to_dev(f["x"], torch.bfloat16)).float().cpu().numpy()
    idx, _ = m._route_tokens(to_dev(f["x"], torch.bfloat16))
    same = (idx.cpu().numpy() == f["topk_idx"]).all(1)
    assert same.mean() > 0.95
    assert max_rel_err(out[same], f["out"][same]) <= 2e-2


def test_bench_records_schema():
    """Records carry every key of the reference driver's schema (+ the stage breakdown)."""
    from swiftmoe_b200.bench_records import run_single_config
    from test_host_logic import REFERENCE_RECORD_KEYS
    r = run_single_config("ultimate", 16, 256, 300, device=torch.device("cuda", 0), enable_profiling=True,
                          warmup=2, iterations=3)
    assert REFERENCE_RECORD_KEYS <= set(r)
    assert {"Router", "Dispatch_Comm", "Expert_Compute", "Combine_Comm"} <= set(r)
    b = run_single_config("baseline", 16, 256, 300, device=torch.device("cuda", 0), warmup=2, iterations=3)
    assert REFERENCE_RECORD_KEYS <= set(b) and b["throughput_tokens_per_sec"] > 0


@torch.no_grad()
def test_fp32_layer_keeps_split_weights(monkeypatch):
    """An fp32 layer passes its routed expert weights pre-split (SMOE_F32_SPLITW): the
    output equals the call that splits them inside the library bit for bit, and after an
    in-place weight update the kept copy is rebuilt (equal again, and different from the
    output before the update)."""
    import swiftmoe_b200 as S
    dev = torch.device("cuda", 0)
    torch.manual_seed(11)
    m = S.UltimateMoE(8, 512, use_fp16=False, dtype=torch.float32, top_k=2, expert_type="swiglu", d_ff=2048,
                      use_nccl_opt=False, device=dev)
    x = torch.randn(777, 512, device=dev)
    kept = m(x)
    assert any(k.endswith("_tf32") for k in m._wcache)
    monkeypatch.setenv("SMOE_FP32_SPLIT_CACHE", "0")
    plain = m(x)
    monkeypatch.delenv("SMOE_FP32_SPLIT_CACHE")
    assert torch.equal(kept, plain)
    m.w2.mul_(1.5)
    kept2 = m(x)
    monkeypatch.setenv("SMOE_FP32_SPLIT_CACHE", "0")
    plain2 = m(x)
    assert torch.equal(kept2, plain2) and not torch.equal(kept, kept2)
