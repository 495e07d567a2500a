"""The peer-copy schedules of the expert-parallel exchange (local-first and chunked) on
gloo CPU ranks, world sizes 2, 4 and 8: the CUDA runtime is replaced by a host double
whose peer buffers are shared-memory segments (tests/p2p_double.py) and the kernels by
the numpy double, so the host bookkeeping (copy segments, buffer layouts, the two-half
split of the own rows, the capacity cut of the own rows, the return addresses of the
fused return, the token dedup) is checked against the oracle's multi-rank forward
without a GPU."""
import ctypes
import os
import zlib
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


def _worker(rank, ws, rdzv, E, d, T, k, cap_factor, schedule, with_shared, result_dir, skew=0.0):
    schedule, *opts = schedule.split("+")
    Ts = list(T) if isinstance(T, (list, tuple)) else [T] * ws     # tokens per rank (ragged)
    T = Ts[rank]
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    import torch.distributed as dist
    import ep_doubles
    from p2p_double import HostRuntime
    from oracle import moe_oracle as O
    from swiftmoe_b200._core import capacity_rows
    from swiftmoe_b200.ep import ExpertParallelExchange
    dist.init_process_group("gloo", init_method=f"file://{rdzv}", rank=rank, world_size=ws)
    rng = np.random.default_rng(0)
    gate = (rng.standard_normal((E, d)) * 0.3).astype(np.float32)
    W = (rng.standard_normal((E, d, d)) * 0.1).astype(np.float32)   # nn.Linear [out, in]
    xs = [np.random.default_rng(10 + r).standard_normal((Ts[r], d)).astype(np.float32) for r in range(ws)]
    x = xs[rank]
    # skew > 0: every token prefers the experts of rank 0 (the other ranks receive nothing)
    bias = np.where(np.arange(E) < E // ws, skew, 0.0).astype(np.float32) if skew else None
    idx, w, _ = O.route(x, gate, k, bias)
    ex = ExpertParallelExchange(E, ws, rank, d, kernels=ep_doubles, chunks=3,
                                transport="p2p", schedule=schedule, runtime=HostRuntime(f"smoet{zlib.crc32(rdzv.encode()):08x}"))
    ex.return_mode = "copy" if "copy" in opts else "fused"
    if "dedup" in opts:
        ex.dedup = "on"
    if "nodedup" in opts:
        ex.dedup = "off"
    cap = capacity_rows(cap_factor, max(Ts), ws, k, E)
    El = E // ws

    def experts(xe, offsets, ends=None, out=None, row_ptrs=None):
        off = offsets.numpy()
        en = off[1:] if ends is None else ends.numpy()
        y = np.zeros((xe.shape[0], d), np.float32) if out is None else out.numpy()
        for le in range(El):
            a, b = int(off[le]), int(en[le])
            if b > a:
                rows = xe.numpy()[a:b] @ W[rank * El + le].T
                if row_ptrs is None:
                    y[a:b] = rows
                    continue
                for i in range(a, b):      # the fused return: rows stored at their addresses
                    p = int(row_ptrs[i])
                    if p:
                        ctypes.memmove(p, np.ascontiguousarray(rows[i - a]).ctypes.data, d * 4)
        return None if row_ptrs is not None else (torch.from_numpy(y) if out is None else out)

    shared = np.random.default_rng(50 + rank).standard_normal((T, d)).astype(np.float32) if with_shared else None
    args = (torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(w), cap, experts)
    kw = dict(shared=None if shared is None else torch.from_numpy(shared))
    # a first batch with other routing leaves other rows in every buffer, so a row the
    # checked batch fails to write shows up as a mismatch
    xo = np.random.default_rng(99 + rank).standard_normal((T, d)).astype(np.float32)
    io, wo, _ = O.route(xo, gate, k, bias)
    ex.forward(torch.from_numpy(xo), torch.from_numpy(io), torch.from_numpy(wo), cap, experts, **kw)
    out1 = ex.forward(*args, **kw).numpy().copy()
    out2 = ex.forward(*args, **kw).numpy().copy()      # buffers reused
    p = O.MoEParams(gate=gate, expert_type="linear", expert_w=np.ascontiguousarray(W.transpose(0, 2, 1)))
    p.logit_bias = bias
    refs, aux = O.moe_forward(xs, p, ws=ws, k=k, capacity=cap, return_aux=True)
    ref = refs[rank] + (shared if shared is not None else 0)
    kept_ref = sum(int(min(cap, c)) if cap > 0 else int(c)
                   for c in np.bincount(np.concatenate([aux["routed"][r][0].ravel() for r in range(ws)]),
                                        minlength=E)[rank * El:(rank + 1) * El])
    err = float(np.abs(out1 - ref).max()) if T else 0.0
    np.save(os.path.join(result_dir, f"err{rank}.npy"),
            np.array([err, float(np.array_equal(out1, out2)), ex.last_rows - kept_ref]))
    ex.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("ws,E,k,cf,schedule,shared", [
    (2, 8, 2, None, "local_first", False), (2, 8, 2, 1.0, "local_first", True),
    (4, 8, 3, None, "local_first", False), (4, 16, 2, 0.5, "local_first", False),
    (8, 8, 2, 0.7, "local_first", False), (8, 16, 2, None, "local_first", True),
    (2, 8, 2, 1.0, "local_first+copy", False), (4, 16, 2, 0.5, "local_first+copy", True),
    (2, 8, 2, 1.0, "chunked", False), (4, 8, 2, 0.5, "chunked", True),
    # token dedup: automatic from k = 4 on, forced at k = 2
    (2, 16, 4, None, "local_first", True), (4, 16, 6, None, "local_first", False),
    (8, 16, 8, None, "local_first", True), (2, 8, 2, None, "local_first+dedup", False),
    (4, 16, 5, 0.5, "local_first", False),
    # device schedule (layout on the device, rows stored into the peers by the send kernel)
    (2, 8, 2, None, "device", False), (2, 8, 2, 1.0, "device", True), (4, 8, 3, None, "device", False),
    (4, 16, 2, 0.5, "device", False), (8, 8, 2, 0.7, "device", False), (8, 16, 2, None, "device", True),
    (4, 16, 5, 0.5, "device", False), (2, 16, 4, None, "device+nodedup", True),
    # device schedule with token dedup (top-k a multiple of 4 with several experts per rank)
    (2, 16, 4, None, "device", True), (4, 16, 8, None, "device", False), (8, 16, 8, None, "device", True)])
def test_p2p_schedules_match_oracle(tmp_path, ws, E, k, cf, schedule, shared):
    T, d = 23, 12
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), E, d, T, k, cf, schedule, shared, str(tmp_path)), nprocs=ws, join=True)
    _check(tmp_path, ws)


@pytest.mark.parametrize("Ts,E,k,cf,schedule", [
    ((0, 23), 8, 2, None, "local_first"), ((5, 0, 23, 1), 8, 2, None, "local_first"),
    ((0, 17), 16, 4, None, "local_first"), ((5, 0, 23, 1), 16, 6, None, "local_first"),
    ((0, 23), 8, 2, 1.0, "local_first"), ((5, 0, 23, 1), 8, 2, 0.5, "chunked"),
    ((0, 23), 8, 2, None, "device"), ((5, 0, 23, 1), 8, 2, 0.5, "device"),
    ((5, 0, 23, 1), 16, 6, None, "device+nodedup"), ((0, 17), 16, 4, None, "device"),
    ((5, 0, 23, 1), 16, 8, None, "device")])
def test_p2p_schedules_ragged_and_empty_batches(tmp_path, Ts, E, k, cf, schedule):
    """Ranks with different token counts, some with none: every rank still takes part in
    every collective step, and the ranks with tokens match the oracle."""
    ws, d = len(Ts), 12
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), E, d, Ts, k, cf, schedule, False, str(tmp_path)), nprocs=ws,
             join=True)
    _check(tmp_path, ws)


def _check(tmp_path, ws):
    for r in range(ws):
        err, same, rows_diff = np.load(tmp_path / f"err{r}.npy")
        assert err <= 1e-5, (r, err)
        assert same == 1.0
        assert rows_diff == 0


@pytest.mark.parametrize("ws,E,k,cf,schedule,skew", [
    (2, 8, 2, None, "local_first", 50.0), (4, 8, 2, 0.5, "local_first", 50.0),
    (4, 16, 4, None, "local_first", 50.0), (4, 8, 8, None, "local_first", 0.0),
    (2, 8, 8, 1.0, "local_first", 0.0), (4, 8, 2, None, "chunked", 50.0),
    (2, 8, 2, None, "device", 50.0), (4, 8, 2, 0.5, "device", 50.0), (4, 8, 8, None, "device+nodedup", 0.0),
    (2, 8, 8, 1.0, "device", 0.0), (4, 16, 4, None, "device", 50.0), (4, 8, 8, None, "device", 0.0)])
def test_p2p_schedules_extreme_routing(tmp_path, ws, E, k, cf, schedule, skew):
    """All tokens routed to one rank's experts (the others compute nothing and receive
    nothing), and k = E (every token to every expert, every rank once with dedup)."""
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), E, 12, 23, k, cf, schedule, False, str(tmp_path), skew),
             nprocs=ws, join=True)
    _check(tmp_path, ws)
