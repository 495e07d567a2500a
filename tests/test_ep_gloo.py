"""Expert-parallel exchange on world-size 2 and 4 gloo CPU ranks (kernels replaced by a
numpy double), against the oracle's multi-rank forward, including capacity drops."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _rdzv(tmp_path):
    """File rendezvous for the spawned ranks (no TCP port that another process can take)."""
    return str(tmp_path / "rendezvous")


def _worker(rank, ws, rdzv, E, d, T, k, cap_factor, chunks, result_dir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch.distributed as dist
    import ep_doubles
    from oracle import moe_oracle as O
    from swiftmoe_b200._core import capacity_rows
    from swiftmoe_b200.ep import ExpertParallelExchange
    dist.init_process_group("gloo", init_method=f"file://{rdzv}", rank=rank, world_size=ws)
    Ts = list(T) if isinstance(T, (list, tuple)) else [T] * ws     # tokens per rank (ragged)
    T = Ts[rank]
    rng = np.random.default_rng(0)
    gate = (rng.standard_normal((E, d)) * 0.3).astype(np.float32)
    W = (rng.standard_normal((E, d, d)) * 0.1).astype(np.float32)   # nn.Linear [out, in]
    xs = [np.random.default_rng(10 + r).standard_normal((Ts[r], d)).astype(np.float32) for r in range(ws)]
    x = xs[rank]
    idx, w, _ = O.route(x, gate, k)
    ex = ExpertParallelExchange(E, ws, rank, d, kernels=ep_doubles, chunks=chunks)
    cap = capacity_rows(cap_factor, max(Ts), ws, k, E)
    El = E // ws

    def experts(xe, offsets):
        off = offsets.numpy()
        y = np.zeros((xe.shape[0], d), np.float32)
        for le in range(El):
            e = rank * El + le
            y[off[le]:off[le + 1]] = xe.numpy()[off[le]:off[le + 1]] @ W[e].T
        return torch.from_numpy(y)

    # chunked, overlapped layer path
    out = ex.forward(torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(w), cap, experts).numpy()
    # unchunked stage API (dispatch / combine)
    xe, offsets, st = ex.dispatch(torch.from_numpy(x), torch.from_numpy(idx), cap)
    out_stage = ex.combine(experts(xe, offsets), st, torch.from_numpy(w)).numpy()
    p = O.MoEParams(gate=gate, expert_type="linear", expert_w=np.ascontiguousarray(W.transpose(0, 2, 1)))
    refs = O.moe_forward(xs, p, ws=ws, k=k, capacity=cap)
    err = max(np.abs(out - refs[rank]).max(), np.abs(out_stage - refs[rank]).max()) if T else 0.0
    np.save(os.path.join(result_dir, f"err{rank}.npy"), np.array([err, out.shape[0] - T]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("ws,E,k,cf,chunks", [(2, 8, 2, None, 1), (2, 8, 2, 1.0, 3), (4, 8, 3, None, 4),
                                               (4, 16, 2, 0.5, 2), (2, 4, 2, 0.7, 5)])
def test_ep_exchange_matches_oracle(tmp_path, ws, E, k, cf, chunks):
    T, d = 23, 12
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), E, d, T, k, cf, chunks, str(tmp_path)), nprocs=ws, join=True)
    for r in range(ws):
        assert float(np.load(tmp_path / f"err{r}.npy")[0]) <= 1e-5


@pytest.mark.parametrize("Ts,E,k,cf,chunks", [((0, 23), 8, 2, None, 3), ((5, 0, 23, 1), 16, 2, 0.5, 4)])
def test_ep_exchange_ragged_and_empty_batches(tmp_path, Ts, E, k, cf, chunks):
    """Ranks with different token counts, some with none: the collective transport's
    per-chunk exchanges still line up on every rank."""
    ws, d = len(Ts), 12
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), E, d, Ts, k, cf, chunks, str(tmp_path)), nprocs=ws, join=True)
    for r in range(ws):
        err, n_diff = np.load(tmp_path / f"err{r}.npy")
        assert err <= 1e-5 and n_diff == 0
