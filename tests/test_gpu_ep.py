"""Expert parallelism on 2+ GPUs (NCCL): the drop-in UltimateMoE on every rank against
the oracle's multi-rank forward (experts split in contiguous blocks, capacity cut in
(source rank, token, slot) order).  Skipped on machines with fewer than two GPUs."""
import datetime
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = Path(__file__).resolve().parent.parent


def _rdzv(tmp_path):
    """File rendezvous for the spawned ranks (no TCP port that another process can take)."""
    return str(tmp_path / "rendezvous")


def _worker(rank, ws, rdzv, cfg, transport, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "tests" / "golden")]
    os.environ.update(LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import synth
    from oracle import moe_oracle as O
    from util import max_rel_err, rounded
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{rdzv}", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    T, d, E, k, F, cf, shared = cfg
    dt = torch.bfloat16
    w1, w3, w2 = synth.swiglu_weights(3, E, d, F, init="normal", std=0.02)
    g = synth.normal(4, (E, d), 0.02)
    sw = synth.swiglu_weights(5, 1, d, F, init="normal", std=0.02) if shared else None
    xs = [rounded(synth.normal(100 + r, (T, d), 1.0), dt) for r in range(ws)]
    import swiftmoe_b200 as S
    m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, expert_type="swiglu", d_ff=F,
                      capacity_factor=cf, num_shared_experts=1 if shared else 0, d_ff_shared=F,
                      use_nccl_opt=False, device=dev)
    tr, _, sched = transport.partition("-")
    tr, *opts = tr.split("+")
    m.comm.transport, m.comm.schedule = tr, sched or "local_first"
    m.comm.return_mode = "copy" if "copy" in opts else "fused"
    if "split" in opts:                   # own rows in two halves even with 2 ranks
        m.comm.split_min_ws = 2
    El = E // ws
    sl = slice(rank * El, (rank + 1) * El)
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(g))
        m.w1.copy_(torch.from_numpy(w1[sl])); m.w3.copy_(torch.from_numpy(w3[sl])); m.w2.copy_(torch.from_numpy(w2[sl]))
        if shared:
            m.shared_w1.copy_(torch.from_numpy(sw[0][0])); m.shared_w3.copy_(torch.from_numpy(sw[1][0]))
            m.shared_w2.copy_(torch.from_numpy(sw[2][0]))
    out = m(torch.from_numpy(xs[rank]).to(dev, dt)).float().cpu().numpy()
    out2 = m(torch.from_numpy(xs[rank]).to(dev, dt)).float().cpu().numpy()   # second call: same bits
    r = lambda a: rounded(a, dt)
    p = O.MoEParams(gate=r(g), expert_type="swiglu", w1=r(w1), w3=r(w3), w2=r(w2))
    if shared:
        p.sw1, p.sw3, p.sw2 = r(sw[0]), r(sw[1]), r(sw[2])
    refs, aux = O.moe_forward(xs, p, ws=ws, k=k, capacity_factor=cf, acc=np.float64, return_aux=True)
    from swiftmoe_b200 import kernels
    same = []
    for rr in range(ws):
        idx, _ = kernels.router(torch.from_numpy(xs[rr]).to(dev, dt), m.gate_weight, k)
        same.append((idx.cpu().numpy() == aux["routed"][rr][0]).all(1))
    if cf is None:
        rows = same[rank]
        err = max_rel_err(out[rows], refs[rank][rows])
    else:
        # with a capacity, a near-tie routing flip on any rank can move the cut; compare
        # only when routing agrees everywhere
        err = max_rel_err(out, refs[rank]) if all(s.all() for s in same) else 0.0
    diff_rows = np.nonzero(np.abs(out - out2).max(1) > 0)[0] if out.size else np.zeros(0, int)
    if diff_rows.size:
        print(f"rank {rank} ({transport}): {diff_rows.size} rows differ between calls, first "
              f"{diff_rows[:8].tolist()}, max |diff| {np.abs(out - out2).max():.3e}", flush=True)
    np.save(os.path.join(out_dir, f"r{rank}.npy"),
            np.array([err, float(np.array_equal(out, out2)), float(same[rank].mean()),
                      float(kernels.read_device_error(dev))]))
    dist.barrier()
    dist.destroy_process_group()


CASES = [(300, 256, 8, 2, 512, None, False), (257, 256, 16, 2, 256, 1.0, False),
         (200, 128, 32, 8, 128, None, True)]


@pytest.mark.parametrize("transport", ["p2p", "p2p+copy", "p2p+split", "p2p-chunked", "collective"])
@pytest.mark.parametrize("cfg", CASES)
def test_ep_layer_matches_oracle(tmp_path, cfg, transport):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    ws = 4 if n >= 4 and cfg[2] % 4 == 0 else 2
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), cfg, transport, str(tmp_path)), nprocs=ws, join=True)
    for r in range(ws):
        err, same_bits, agree, dev_err = np.load(tmp_path / f"r{r}.npy")
        assert dev_err == 0.0
        assert agree > 0.99
        assert err <= 2e-2, (r, err)
        assert same_bits == 1.0


def _ref_fixture_worker(rank, ws, rdzv, name, transport, out_dir):
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
    m = S.UltimateMoE(E, d, use_fp16=False, use_nccl_opt=False).to(dev)
    m.comm.transport = transport
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(p.gate))
        m.expert_weights.copy_(torch.from_numpy(p.expert_w[rank * El:(rank + 1) * El]))
    out = m(torch.from_numpy(f["x"][rank]).to(dev)).cpu().numpy()
    err = float(np.abs(out - f["out"][rank]).max())
    np.save(os.path.join(out_dir, f"ref{rank}.npy"), np.array([err]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["p2p", "collective"])
@pytest.mark.parametrize("name,ws", [("ult_linear_fp32_ws2_E8_d32_M23", 2), ("ult_linear_fp32_ws4_E8_d32_M17", 4)])
def test_ep_matches_reference_ultimate_moe(tmp_path, name, ws, transport):
    """fp32 UltimateMoE over `ws` GPUs against the reference's own UltimateMoE run with the
    same world size (gloo, CPU): max-abs 1e-5 on every rank."""
    if torch.cuda.device_count() < ws:
        pytest.skip(f"needs {ws} GPUs")
    mp.spawn(_ref_fixture_worker, args=(ws, _rdzv(tmp_path), name, transport, str(tmp_path)), nprocs=ws, join=True)
    for r in range(ws):
        assert float(np.load(tmp_path / f"ref{r}.npy")[0]) <= 1e-5
