"""Expert parallelism on 2, 4 and 8 GPUs (NCCL): the drop-in UltimateMoE on every rank
against the oracle's multi-rank forward (experts split in contiguous blocks, capacity
cut in (source rank, token, slot) order), for every exchange schedule.

Parity is checked on two levels, so that no case passes without a comparison:
* routing: the GPU router's expert choices against the oracle's router on the same
  rounded inputs -- every disagreement must be a near-tie of the oracle's logits;
* the layer: every output row against the oracle's multi-rank forward run on the
  GPU's own routing (gathered from all ranks), so dispatch, capacity cut, experts,
  return and combine are compared on every row, capacity cases included
  (bf16 tolerance: max|out - ref| / max|ref| <= 2e-2).
Each world size runs all its cases in one set of rank processes.  Skipped on machines
with fewer GPUs than the world size."""
import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = Path(__file__).resolve().parent.parent

# name -> (tokens per rank, d_model, experts, top-k, d_ff, capacity factor, shared expert,
#          std of the per-expert router offsets)
CASES = {
    "mixtral-like": (300, 256, 8, 2, 512, None, False, 0.0),
    "capacity": (257, 256, 16, 2, 256, 1.0, False, 0.0),
    "k8-shared": (200, 128, 32, 8, 128, None, True, 0.0),
    # the capacity-limited expert-parallel layer's shape: 64 experts, top-2, d_model 4096,
    # capacity factor 1.25 (d_ff reduced so that the oracle finishes in seconds)
    "ep-capacity-shape": (192, 4096, 64, 2, 128, 1.25, False, 0.0),
    # the fine-grained layer's shape: 128 experts + 1 shared, top-8, d_model 2048, router
    # offsets ~ N(0, 1.5) for load imbalance (d_ff reduced)
    "fine-grained-shape": (160, 2048, 128, 8, 128, None, True, 1.5),
}
# "p2p" = the default schedule (device-side layout, rows stored into the peers by the
# send kernel); the host-laid-out schedules and the collective transport stay selectable
TRANSPORTS = ["p2p", "p2p-local_first", "p2p+copy-local_first", "p2p+split-local_first", "p2p-chunked",
              "collective"]
# SMOE_EP_TEST_TRANSPORTS=a,b,... runs a subset (machines billed per GPU-minute)
if os.environ.get("SMOE_EP_TEST_TRANSPORTS"):
    TRANSPORTS = [t for t in os.environ["SMOE_EP_TEST_TRANSPORTS"].split(",") if t in TRANSPORTS]


def _rdzv(tmp_path):
    """File rendezvous for the spawned ranks (no TCP port that another process can take)."""
    return str(tmp_path / "rendezvous")


def _configure(m, transport):
    tr, _, sched = transport.partition("-")
    tr, *opts = tr.split("+")
    m.comm.transport, m.comm.schedule = tr, sched or "device"
    m.comm.return_mode = "copy" if "copy" in opts else "fused"
    if "split" in opts:                   # own rows in two halves even with 2 ranks
        m.comm.split_min_ws = 2


_ORACLE = {}   # (case, routing digest) -> this rank's oracle rows: one oracle run per case


def _run_case(rank, ws, dev, case, transport):
    import torch.distributed as dist
    import synth
    from oracle import moe_oracle as O
    from util import elementwise_rel_err, max_rel_err, rounded, routing_matches_up_to_ties
    import swiftmoe_b200 as S
    from swiftmoe_b200 import kernels
    T, d, E, k, F, cf, shared, bias_std = case
    dt = torch.bfloat16
    w1, w3, w2 = synth.swiglu_weights(3, E, d, F, init="normal", std=0.02)
    g = synth.normal(4, (E, d), 0.02)
    bias = synth.normal(6, (E,), bias_std) if bias_std else None
    sw = synth.swiglu_weights(5, 1, d, F, init="normal", std=0.02) if shared else None
    xs = [rounded(synth.normal(100 + r, (T, d), 1.0), dt) for r in range(ws)]
    m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, expert_type="swiglu", d_ff=F,
                      capacity_factor=cf, num_shared_experts=1 if shared else 0, d_ff_shared=F,
                      use_nccl_opt=False, device=dev)
    _configure(m, transport)
    El = E // ws
    sl = slice(rank * El, (rank + 1) * El)
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(g))
        m.w1.copy_(torch.from_numpy(w1[sl])); m.w3.copy_(torch.from_numpy(w3[sl])); m.w2.copy_(torch.from_numpy(w2[sl]))
        if shared:
            m.shared_w1.copy_(torch.from_numpy(sw[0][0])); m.shared_w3.copy_(torch.from_numpy(sw[1][0]))
            m.shared_w2.copy_(torch.from_numpy(sw[2][0]))
    if bias is not None:
        m.set_logit_bias(torch.from_numpy(bias))
    x = torch.from_numpy(xs[rank]).to(dev, dt)
    with torch.no_grad():
        out = m(x).float().cpu().numpy()
        out2 = m(x).float().cpu().numpy()      # second call: same bits
    # every rank's routing, as the GPU computed it
    idx, w = kernels.router(x, m.gate_weight, k, m.logit_bias)
    all_idx = [torch.empty_like(idx) for _ in range(ws)]
    all_w = [torch.empty_like(w) for _ in range(ws)]
    dist.all_gather(all_idx, idx)
    dist.all_gather(all_w, w)
    routing = [(a.cpu().numpy(), b.cpu().numpy()) for a, b in zip(all_idx, all_w)]
    dev_err = int(kernels.read_device_error(dev))
    m.comm.close()                             # collective: frees this layer's peer buffers
    r = lambda a: rounded(a, dt)
    p = O.MoEParams(gate=r(g), expert_type="swiglu", w1=r(w1), w3=r(w3), w2=r(w2))
    p.logit_bias = bias
    if shared:
        p.sw1, p.sw3, p.sw2 = r(sw[0]), r(sw[1]), r(sw[2])
    import hashlib
    key = (case, hashlib.sha1(b"".join(a.tobytes() + b.tobytes() for a, b in routing)).hexdigest())
    if key not in _ORACLE:
        _ORACLE[key] = O.moe_forward(xs, p, ws=ws, k=k, capacity_factor=cf, acc=np.float32, routing=routing)[rank]
    ref = _ORACLE[key]
    # routing against the oracle's own router: differences only at near-ties
    o_idx, _, logits = O.route(xs[rank], p.gate, k, p.logit_bias)
    own = routing[rank][0]
    tie_bad = routing_matches_up_to_ties(own, o_idx, logits, rtol=1e-4)
    return dict(err=max_rel_err(out, ref), elem=elementwise_rel_err(out, ref), rows=int(out.shape[0]),
                same_bits=bool(np.array_equal(out, out2)), agree=float((own == o_idx).all(1).mean()),
                tie_bad=len(tie_bad), dev_err=dev_err)


def _worker(rank, ws, rdzv, cases, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "tests" / "golden")]
    os.environ.update(LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{rdzv}", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    results = {}
    for name, transport in cases:
        results[f"{name}/{transport}"] = _run_case(rank, ws, dev, CASES[name], transport)
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
        json.dump(results, f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("ws", [2, 4, 8])
def test_ep_layer_matches_oracle(tmp_path, ws):
    if torch.cuda.device_count() < ws:
        pytest.skip(f"needs {ws} GPUs")
    cases = [(n, t) for n in CASES for t in TRANSPORTS]
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), cases, str(tmp_path)), nprocs=ws, join=True)
    bad = []
    for r in range(ws):
        res = json.loads((tmp_path / f"r{r}.json").read_text())
        for key, v in res.items():
            print(f"ws={ws} rank {r} {key}: max-rel {v['err']:.2e} (element-wise {v['elem']:.2e}) over "
                  f"{v['rows']} rows, routing agreement {v['agree']:.4f}")
            if v["dev_err"] != 0 or v["err"] > 2e-2 or not v["same_bits"] or v["tie_bad"] or v["rows"] == 0:
                bad.append((r, key, v))
    assert not bad, bad


def _ref_fixture_worker(rank, ws, rdzv, name, transports, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "tests" / "golden")]
    os.environ.update(LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import fixtures as fx
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{rdzv}", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    import swiftmoe_b200 as S
    f, p = fx.ult_linear(name)
    E, d = f["E"], f["d"]
    El = E // ws
    errs = []
    for transport in transports:
        m = S.UltimateMoE(E, d, use_fp16=False, use_nccl_opt=False).to(dev)
        _configure(m, transport)
        with torch.no_grad():
            m.gate_weight.copy_(torch.from_numpy(p.gate))
            m.expert_weights.copy_(torch.from_numpy(p.expert_w[rank * El:(rank + 1) * El]))
        with torch.no_grad():
            out = m(torch.from_numpy(f["x"][rank]).to(dev)).cpu().numpy()
        errs.append(float(np.abs(out - f["out"][rank]).max()))
        m.comm.close()
    np.save(os.path.join(out_dir, f"ref{rank}.npy"), np.array(errs))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name,ws", [("ult_linear_fp32_ws2_E8_d32_M23", 2), ("ult_linear_fp32_ws4_E8_d32_M17", 4)])
def test_ep_matches_reference_ultimate_moe(tmp_path, name, ws):
    """fp32 UltimateMoE over `ws` GPUs against the reference's own UltimateMoE run with the
    same world size (gloo, CPU): max-abs 1e-5 on every rank, every transport."""
    if torch.cuda.device_count() < ws:
        pytest.skip(f"needs {ws} GPUs")
    mp.spawn(_ref_fixture_worker, args=(ws, _rdzv(tmp_path), name, TRANSPORTS, str(tmp_path)), nprocs=ws,
             join=True)
    for r in range(ws):
        errs = np.load(tmp_path / f"ref{r}.npy")
        assert float(errs.max()) <= 1e-5, dict(zip(TRANSPORTS, errs.tolist()))
