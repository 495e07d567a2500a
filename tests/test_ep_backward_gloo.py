"""Expert-parallel layer backward (``ExpertParallelExchange.layer_backward``) on world-size
2 and 4 gloo CPU ranks, kernels replaced by the numpy double, against the oracle's
backward of the whole batch (expert parallelism only moves rows: each rank's input
gradient is the whole-batch gradient of its tokens, each rank's local experts get the
whole-batch gradient of those experts, and the replicated gate / shared expert get their
whole-batch gradient as the sum of the ranks' contributions).  SwiGLU and linear experts,
capacity drops, a shared expert and router offsets."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _rdzv(tmp_path):
    return str(tmp_path / "rendezvous")


def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def _worker(rank, ws, rdzv, E, d, F, T, k, cf, kind, with_shared, with_bias, result_dir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch.distributed as dist
    import ep_doubles
    from oracle import moe_oracle as O
    from swiftmoe_b200._core import capacity_rows
    from swiftmoe_b200.ep import ExpertParallelExchange
    dist.init_process_group("gloo", init_method=f"file://{rdzv}", rank=rank, world_size=ws)
    rng = np.random.default_rng(0)
    f = np.float32
    gate = (rng.standard_normal((E, d)) * 0.3).astype(f)
    bias = (rng.standard_normal(E) * 1.5).astype(f) if with_bias else None
    xs = [np.random.default_rng(10 + r).standard_normal((T, d)).astype(f) for r in range(ws)]
    dos = [np.random.default_rng(50 + r).standard_normal((T, d)).astype(f) for r in range(ws)]
    El = E // ws
    sl = slice(rank * El, (rank + 1) * El)
    t = torch.from_numpy
    p = O.MoEParams(gate=gate, expert_type=kind, logit_bias=bias)
    if kind == "swiglu":
        w1 = (rng.standard_normal((E, F, d)) * 0.2).astype(f)
        w3 = (rng.standard_normal((E, F, d)) * 0.2).astype(f)
        w2 = (rng.standard_normal((E, d, F)) * 0.2).astype(f)
        p.w1, p.w3, p.w2 = w1, w3, w2
        experts = dict(kind="swiglu", w1=t(w1[sl]), w3=t(w3[sl]), w2t=t(w2[sl]).transpose(1, 2).contiguous(),
                       w13t=t(np.concatenate([w1[sl], w3[sl]], 1)).transpose(1, 2).contiguous())
    else:
        W = (rng.standard_normal((E, d, d)) * 0.2).astype(f)          # x @ W layout
        p.expert_w = W
        experts = dict(kind="linear", w=t(W[sl]).contiguous(), transposed=True)
    sh = None
    if with_shared:
        Fs = F
        sw1 = (rng.standard_normal((1, Fs, d)) * 0.2).astype(f)
        sw3 = (rng.standard_normal((1, Fs, d)) * 0.2).astype(f)
        sw2 = (rng.standard_normal((1, d, Fs)) * 0.2).astype(f)
        p.sw1, p.sw3, p.sw2 = sw1, sw3, sw2
        sh = dict(w1=t(sw1), w3=t(sw3), w2t=t(sw2).transpose(1, 2).contiguous(),
                  w13t=t(np.concatenate([sw1, sw3], 1)).transpose(1, 2).contiguous())
    ex = ExpertParallelExchange(E, ws, rank, d, kernels=ep_doubles)
    cap = capacity_rows(cf, T, ws, k, E)
    g = ex.layer_backward(t(xs[rank]), t(dos[rank]), t(gate), t(bias) if bias is not None else None, k, cap,
                          experts, sh)
    ref = O.moe_backward(np.concatenate(xs), p, np.concatenate(dos), k=k, capacity=cap or None, acc=np.float64)
    err = {"x": _rel(g["x"].numpy(), ref["x"][rank * T:(rank + 1) * T])}
    if kind == "swiglu":
        err["w1"] = _rel(g["w13"][:, :F].numpy(), ref["w1"][sl])
        err["w3"] = _rel(g["w13"][:, F:].numpy(), ref["w3"][sl])
        err["w2"] = _rel(g["w2"].numpy(), ref["w2"][sl])
    else:
        err["expert_w"] = _rel(g["lin"].numpy(), ref["expert_w"][sl])
    gg = g["gate"].clone()
    dist.all_reduce(gg)
    err["gate"] = _rel(gg.numpy(), ref["gate"])
    if sh is not None:
        s13, s2 = g["s13"].clone(), g["s2"].clone()
        dist.all_reduce(s13)
        dist.all_reduce(s2)
        err["sw1"] = _rel(s13[:F].numpy(), ref["sw1"][0])
        err["sw3"] = _rel(s13[F:].numpy(), ref["sw3"][0])
        err["sw2"] = _rel(s2.numpy(), ref["sw2"][0])
    np.save(os.path.join(result_dir, f"err{rank}.npy"), np.array([max(err.values())]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("ws,E,k,cf,kind,shared,bias", [
    (2, 8, 2, None, "swiglu", False, False),
    (2, 8, 2, 0.8, "swiglu", True, True),       # capacity drops, shared expert, router offsets
    (4, 8, 4, None, "swiglu", True, False),
    (4, 16, 2, 0.6, "linear", False, True),
    (2, 4, 2, None, "linear", True, False),
])
def test_ep_backward_matches_whole_batch_oracle(tmp_path, ws, E, k, cf, kind, shared, bias):
    T, d, F = 19, 16, 24
    mp.spawn(_worker, args=(ws, _rdzv(tmp_path), E, d, F, T, k, cf, kind, shared, bias, str(tmp_path)),
             nprocs=ws, join=True)
    for r in range(ws):
        assert float(np.load(tmp_path / f"err{r}.npy")[0]) <= 1e-4
