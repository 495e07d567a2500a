"""Expert-parallel layer backward on 2 and 4 GPUs (NCCL): ``UltimateMoE`` under autograd on
every rank against the oracle's backward of the whole batch on the GPUs' own routing
(gathered from all ranks).  Expert parallelism only moves rows, so each rank's input
gradient is the whole-batch gradient of its tokens and its local experts' gradients the
whole-batch gradients of those experts; the replicated gate and shared expert get their
whole-batch gradient as the sum of the ranks' contributions.  bf16 tolerance: max|g -
ref| / max|ref| <= 2e-2 per gradient, as for the one-GPU backward."""
import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu, pytest.mark.autograd]
ROOT = Path(__file__).resolve().parent.parent

# name -> (tokens per rank, d_model, experts, top-k, d_ff (0: linear experts), capacity factor,
#          shared expert, std of the router offsets)
CASES = {
    "swiglu": (200, 256, 8, 2, 256, None, False, 0.0),
    "swiglu-capacity-shared": (160, 128, 16, 2, 128, 1.0, True, 1.5),
    "swiglu-k4": (128, 128, 8, 4, 128, None, False, 0.0),
    "linear": (150, 128, 8, 2, 0, None, False, 0.0),
}


def _run_case(rank, ws, dev, case):
    import torch.distributed as dist
    import synth
    from oracle import moe_oracle as O
    from util import max_rel_err, rounded
    import swiftmoe_b200 as S
    from swiftmoe_b200 import kernels
    from swiftmoe_b200._core import capacity_rows
    T, d, E, k, F, cf, shared, bias_std = case
    dt = torch.bfloat16
    r = lambda a: rounded(a, dt)
    El = E // ws
    sl = slice(rank * El, (rank + 1) * El)
    gw = synth.normal(4, (E, d), 0.1)
    bias = synth.normal(6, (E,), bias_std) if bias_std else None
    xs = [r(synth.normal(100 + q, (T, d), 1.0)) for q in range(ws)]
    dos = [r(synth.normal(200 + q, (T, d), 1.0)) for q in range(ws)]
    if F:
        w1, w3, w2 = synth.swiglu_weights(3, E, d, F, init="normal", std=0.05)
        m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, expert_type="swiglu", d_ff=F,
                          capacity_factor=cf, num_shared_experts=1 if shared else 0, d_ff_shared=F,
                          use_nccl_opt=False, device=dev)
        p = O.MoEParams(gate=r(gw), expert_type="swiglu", w1=r(w1), w3=r(w3), w2=r(w2))
        with torch.no_grad():
            m.w1.copy_(torch.from_numpy(w1[sl])); m.w3.copy_(torch.from_numpy(w3[sl]))
            m.w2.copy_(torch.from_numpy(w2[sl]))
    else:
        W = synth.normal(7, (E, d, d), 0.05)
        m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, capacity_factor=cf, use_nccl_opt=False,
                          device=dev)
        p = O.MoEParams(gate=r(gw), expert_type="linear", expert_w=r(W))
        with torch.no_grad():
            m.expert_weights.copy_(torch.from_numpy(W[sl]))
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(gw))
    if shared:
        sw = synth.swiglu_weights(5, 1, d, F, init="normal", std=0.05)
        p.sw1, p.sw3, p.sw2 = r(sw[0]), r(sw[1]), r(sw[2])
        with torch.no_grad():
            m.shared_w1.copy_(torch.from_numpy(sw[0][0])); m.shared_w3.copy_(torch.from_numpy(sw[1][0]))
            m.shared_w2.copy_(torch.from_numpy(sw[2][0]))
    if bias is not None:
        m.set_logit_bias(torch.from_numpy(bias))
        p.logit_bias = bias
    x = torch.from_numpy(xs[rank]).to(dev, dt).requires_grad_(True)
    m(x).backward(torch.from_numpy(dos[rank]).to(dev, dt))
    # every rank's routing, as the GPU computed it
    idx, w = kernels.router(x.detach(), m.gate_weight.detach(), k, m.logit_bias)
    all_idx = [torch.empty_like(idx) for _ in range(ws)]
    all_w = [torch.empty_like(w) for _ in range(ws)]
    dist.all_gather(all_idx, idx)
    dist.all_gather(all_w, w)
    routing = (np.concatenate([a.cpu().numpy() for a in all_idx]), np.concatenate([b.cpu().numpy() for b in all_w]))
    cap = capacity_rows(cf, T, ws, k, E)
    ref = O.moe_backward(np.concatenate(xs), p, np.concatenate(dos), k=k, capacity=cap or None, routing=routing)
    err = {"x": max_rel_err(x.grad.float().cpu().numpy(), ref["x"][rank * T:(rank + 1) * T])}
    gate_g = m.gate_weight.grad.float().clone()
    dist.all_reduce(gate_g)                      # replicated weight: the ranks' contributions add up
    err["gate"] = max_rel_err(gate_g.cpu().numpy(), ref["gate"])
    if F:
        for n in ("w1", "w3", "w2"):
            err[n] = max_rel_err(getattr(m, n).grad.float().cpu().numpy(), ref[n][sl])
    else:
        err["expert_w"] = max_rel_err(m.expert_weights.grad.float().cpu().numpy(), ref["expert_w"][sl])
    if shared:
        for n, prm in (("sw1", m.shared_w1), ("sw3", m.shared_w3), ("sw2", m.shared_w2)):
            gs = prm.grad.float().clone()
            dist.all_reduce(gs)
            err[n] = max_rel_err(gs.cpu().numpy(), ref[n][0])
    err["dev_err"] = float(kernels.read_device_error(dev))
    m.comm.close()
    return err


def _worker(rank, ws, rdzv, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "tests" / "golden")]
    os.environ.update(LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{rdzv}", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    res = {name: _run_case(rank, ws, dev, case) for name, case in CASES.items()}
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("ws", [2, 4])
def test_ep_backward_matches_whole_batch_oracle(tmp_path, ws):
    if torch.cuda.device_count() < ws:
        pytest.skip(f"needs {ws} GPUs")
    mp.spawn(_worker, args=(ws, str(tmp_path / "rendezvous"), str(tmp_path)), nprocs=ws, join=True)
    bad = []
    for r in range(ws):
        res = json.loads((tmp_path / f"r{r}.json").read_text())
        for name, e in res.items():
            print(f"ws={ws} rank {r} {name}: " + ", ".join(f"{n} {v:.2e}" for n, v in e.items()))
            if e.pop("dev_err") != 0 or max(e.values()) > 2e-2:
                bad.append((r, name, e))
    assert not bad, bad


def _ws1_worker(rank, rdzv, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "tests" / "golden")]
    import torch.distributed as dist
    import synth
    from util import max_rel_err
    import swiftmoe_b200 as S
    from swiftmoe_b200 import kernels
    from swiftmoe_b200.ep import ExpertParallelExchange
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"file://{rdzv}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    res = {}
    for name, (T, d, E, k, F, cf, shared, bias_std) in CASES.items():
        torch.manual_seed(0)
        dt = torch.bfloat16
        if F:
            m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, expert_type="swiglu", d_ff=F,
                              capacity_factor=cf, num_shared_experts=1 if shared else 0, d_ff_shared=F,
                              use_nccl_opt=False, device=dev, init_std=0.05)
        else:
            m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, capacity_factor=cf, use_nccl_opt=False,
                              device=dev, init_std=0.05)
        if bias_std:
            m.set_logit_bias(torch.from_numpy(synth.normal(6, (E,), bias_std)))
        x = torch.from_numpy(synth.normal(100, (T, d), 1.0)).to(dev, dt)
        dout = torch.from_numpy(synth.normal(200, (T, d), 1.0)).to(dev, dt)
        ref = m._backward_fused(x, dout)                 # the one-call backward (smoe_layer_bwd)
        m.comm = ExpertParallelExchange(E, 1, 0, d)      # the expert-parallel pieces, one rank
        got = m._backward_ep(x, dout)
        res[name] = {n: max_rel_err(got[n].float().cpu().numpy(), ref[n].float().cpu().numpy()) for n in ref}
        res[name]["dev_err"] = float(kernels.read_device_error(dev))
    with open(os.path.join(out_dir, "ws1.json"), "w") as f:
        json.dump(res, f)
    dist.destroy_process_group()


def test_ep_backward_pieces_match_fused_backward_on_one_gpu(tmp_path):
    """``layer_backward`` (the expert-parallel split: routed rows on their experts' rank,
    tokens on theirs) on a one-rank group against ``smoe_layer_bwd`` on the same layer:
    every gradient within 1e-2 (bf16, different grouping of the same sums)."""
    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    mp.spawn(_ws1_worker, args=(str(tmp_path / "rendezvous"), str(tmp_path)), nprocs=1, join=True)
    res = json.loads((tmp_path / "ws1.json").read_text())
    bad = []
    for name, e in res.items():
        print(name, ", ".join(f"{n} {v:.2e}" for n, v in e.items()))
        if e.pop("dev_err") != 0 or max(e.values()) > 1e-2:
            bad.append((name, e))
    assert not bad, bad
