"""Generate golden fixtures by running the SwiftMoE reference itself on the CPU.

Run from the repository root in a container where the reference checkout exists:

    python tests/golden/make_golden.py /root/reference          # every fixture
    python tests/golden/make_golden.py /root/reference grads    # gradient fixtures only

It imports ``models.baseline_moe.StandardMoE`` and ``models.ultimate_moe.UltimateMoE``
from that checkout, loads seeded weights into them through their own parameter names,
runs their unmodified ``forward`` (the torch paths: ``StandardMoE`` without a process
group, ``UltimateMoE(use_triton=False)`` under a gloo group of world size 1 or 2) and
stores inputs and outputs as small ``.npz`` files next to this script.  Weights are not
stored: each fixture records its seed in ``meta`` and ``synth.py`` regenerates them
(gate ``normal(seed,(E,d),0.02)``, linear experts ``normal(seed+1,(E,d,d),0.02)``,
SwiGLU ``swiglu_weights(seed,...)`` and gate ``xavier_normal(seed+5,(E,d))``).

The reference has no SwiGLU expert; the ``swiglu`` fixtures substitute SwiGLU modules
into ``StandardMoE.experts`` so that the reference's own route / dispatch / combine
code (``models/baseline_moe.py:56-189``) runs around them.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import synth  # noqa: E402


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _swiglu_module(torch, nn, w1, w3, w2):
    class SwiGLU(nn.Module):
        def __init__(self):
            super().__init__()
            F_, d_ = w1.shape
            self.w1 = nn.Linear(d_, F_, bias=False)
            self.w3 = nn.Linear(d_, F_, bias=False)
            self.w2 = nn.Linear(F_, d_, bias=False)
            with torch.no_grad():
                self.w1.weight.copy_(torch.from_numpy(w1))
                self.w3.weight.copy_(torch.from_numpy(w3))
                self.w2.weight.copy_(torch.from_numpy(w2))

        def forward(self, x):
            return self.w2(torch.nn.functional.silu(self.w1(x)) * self.w3(x))
    return SwiGLU()


def standard_linear(torch, StandardMoE, name, E, d, M, seed, fp16=False):
    g = synth.normal(seed, (E, d), 0.02)
    W = synth.normal(seed + 1, (E, d, d), 0.02)          # nn.Linear weight [out, in]
    x = synth.normal(seed + 2, (M, d), 1.0)
    m = StandardMoE(num_experts=E, d_model=d, use_fp16=fp16)
    dt = torch.float16 if fp16 else torch.float32
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy(g).to(dt))
        for i in range(E):
            m.experts[i].weight.copy_(torch.from_numpy(W[i]).to(dt))
        xt = torch.from_numpy(x).to(dt)
        logits = m.gate(xt)
        idx, w = m._route_tokens(xt)
        out = m(xt)
    np.savez_compressed(HERE / f"{name}.npz", x=x,
                        logits=logits.float().numpy(), topk_idx=idx.int().numpy(),
                        topk_w=w.float().numpy(), out=out.float().numpy(),
                        meta=np.array([E, d, M, seed, int(fp16)]))


def standard_swiglu(torch, nn, StandardMoE, name, E, d, F, M, seed, x_only_seed=None):
    w1, w3, w2 = synth.swiglu_weights(seed, E, d, F, init="xavier")
    g = synth.xavier_normal(seed + 5, (E, d))
    x = synth.normal(seed + 7 if x_only_seed is None else x_only_seed, (M, d), 1.0)
    m = StandardMoE(num_experts=E, d_model=d, use_fp16=False)
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy(g))
    m.experts = nn.ModuleList([_swiglu_module(torch, nn, w1[i], w3[i], w2[i]) for i in range(E)])
    with torch.no_grad():
        xt = torch.from_numpy(x)
        idx, w = m._route_tokens(xt)
        out = m(xt)
    np.savez_compressed(HERE / f"{name}.npz", x=x, topk_idx=idx.int().numpy(),
                        topk_w=w.float().numpy(), out=out.float().numpy(),
                        meta=np.array([E, d, F, M, seed, -1 if x_only_seed is None else x_only_seed]))


def standard_swiglu_lowp(torch, nn, StandardMoE, name, E, d, F, M, seed, dtype_name):
    """The reference's StandardMoE run in a 16-bit dtype with SwiGLU experts substituted:
    its own low-precision output, for comparing a 16-bit implementation against it."""
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype_name]
    w1, w3, w2 = synth.swiglu_weights(seed, E, d, F, init="normal", std=0.02)
    g = synth.normal(seed + 5, (E, d), 0.02)
    x = synth.normal(seed + 7, (M, d), 1.0)
    m = StandardMoE(num_experts=E, d_model=d, use_fp16=False)
    m.experts = nn.ModuleList([_swiglu_module(torch, nn, w1[i], w3[i], w2[i]) for i in range(E)])
    m = m.to(dt)
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy(g))
        xt = torch.from_numpy(x).to(dt)
        idx, w = m._route_tokens(xt)
        out = m(xt)
    np.savez_compressed(HERE / f"{name}.npz", x=xt.float().numpy(), topk_idx=idx.int().numpy(),
                        out=out.float().numpy(), meta=np.array([E, d, F, M, seed]))


def _ult_worker(rank, ws, port, ref, E, d, M, seed, out_path):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ref)
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    import warnings
    warnings.simplefilter("ignore")
    from models.ultimate_moe import UltimateMoE
    g = synth.normal(seed, (E, d), 0.02)
    W = synth.normal(seed + 1, (E, d, d), 0.02)            # x @ W layout
    el = E // ws
    m = UltimateMoE(num_experts=E, d_model=d, use_fp16=False, use_triton=False,
                    use_nccl_opt=False)
    x = synth.normal(seed + 100 + rank, (M, d), 1.0)
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(g))
        m.expert_weights.copy_(torch.from_numpy(W[rank * el:(rank + 1) * el]))
        out = m(torch.from_numpy(x))
    np.savez_compressed(out_path.format(rank=rank), x=x, out=out.numpy())
    dist.barrier()
    dist.destroy_process_group()


def ultimate_linear(name, ref, E, d, M, seed, ws):
    import torch.multiprocessing as mp
    port = _free_port()
    tmp = str(HERE / f"_{name}_r{{rank}}.npz")
    mp.spawn(_ult_worker, args=(ws, port, ref, E, d, M, seed, tmp), nprocs=ws, join=True)
    parts = [np.load(tmp.format(rank=r)) for r in range(ws)]
    np.savez_compressed(HERE / f"{name}.npz",
                        x=np.stack([p["x"] for p in parts]), out=np.stack([p["out"] for p in parts]),
                        meta=np.array([E, d, M, seed, ws]))
    for r in range(ws):
        os.remove(tmp.format(rank=r))


def topk_ties(torch, name, seed):
    """Tie-heavy logits and bf16-rounded logits with torch.topk's values (ties as torch)."""
    rng = np.random.default_rng(seed)
    cases = {}
    for E, k in [(8, 2), (64, 2), (64, 8), (128, 8), (256, 2), (7, 3)]:
        ints = rng.integers(-4, 4, size=(96, E)).astype(np.float32)
        real = (rng.standard_normal((96, E)) * 1.5).astype(np.float32)
        bf = torch.from_numpy(real).bfloat16().float().numpy()
        for tag, lg in (("int", ints), ("real", real), ("bf16", bf)):
            v, i = torch.topk(torch.from_numpy(lg), k, dim=-1)
            cases[f"E{E}_k{k}_{tag}_logits"] = lg
            cases[f"E{E}_k{k}_{tag}_vals"] = v.numpy()
            cases[f"E{E}_k{k}_{tag}_idx"] = i.int().numpy()
            cases[f"E{E}_k{k}_{tag}_w"] = torch.softmax(v, dim=-1).numpy()
    np.savez_compressed(HERE / f"{name}.npz", **cases)


def standard_grads(torch, nn, StandardMoE, name, kind, E, d, F, M, seed):
    """Gradients of the reference's StandardMoE (fp32, no process group) for a seeded
    upstream gradient: its forward is torch ops end to end, so autograd differentiates
    the reference's own route / dispatch / combine code (the reference itself is
    forward-only).  ``kind`` "linear" or "swiglu" (SwiGLU modules substituted)."""
    m = StandardMoE(num_experts=E, d_model=d, use_fp16=False)
    if kind == "linear":
        g = synth.normal(seed, (E, d), 0.02)
        W = synth.normal(seed + 1, (E, d, d), 0.02)
        with torch.no_grad():
            for i in range(E):
                m.experts[i].weight.copy_(torch.from_numpy(W[i]))
    else:
        w1, w3, w2 = synth.swiglu_weights(seed, E, d, F, init="xavier")
        g = synth.xavier_normal(seed + 5, (E, d))
        m.experts = nn.ModuleList([_swiglu_module(torch, nn, w1[i], w3[i], w2[i]) for i in range(E)])
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy(g))
    x = synth.normal(seed + 2, (M, d), 1.0)
    dout = synth.normal(seed + 3, (M, d), 1.0)
    xt = torch.from_numpy(x).requires_grad_(True)
    out = m(xt)
    out.backward(torch.from_numpy(dout))
    grads = dict(dx=xt.grad.numpy(), dgate=m.gate.weight.grad.numpy())
    if kind == "linear":
        grads["dexpert"] = np.stack([m.experts[i].weight.grad.numpy() for i in range(E)])   # [out, in]
    else:
        for n in ("w1", "w3", "w2"):
            grads["d" + n] = np.stack([getattr(m.experts[i], n).weight.grad.numpy() for i in range(E)])
    np.savez_compressed(HERE / f"{name}.npz", x=x, dout=dout, out=out.detach().numpy(),
                        meta=np.array([E, d, F, M, seed, int(kind == "swiglu")]), **grads)


def main(ref: str, only=None):
    sys.path.insert(0, ref)
    import warnings
    warnings.simplefilter("ignore")
    import torch
    import torch.nn as nn
    torch.set_num_threads(4)
    from models.baseline_moe import StandardMoE

    if only == "grads":
        grads_fixtures(torch, nn, StandardMoE)
        return
    standard_linear(torch, StandardMoE, "std_linear_fp32_E8_d64_M37", 8, 64, 37, 11)
    standard_linear(torch, StandardMoE, "std_linear_fp32_E16_d128_M1", 16, 128, 1, 12)
    standard_linear(torch, StandardMoE, "std_linear_fp32_E8_d64_M0", 8, 64, 0, 13)
    standard_linear(torch, StandardMoE, "std_linear_fp32_E64_d256_M300", 64, 256, 300, 14)
    standard_linear(torch, StandardMoE, "std_linear_fp16_E8_d128_M33", 8, 128, 33, 15, fp16=True)
    standard_swiglu(torch, nn, StandardMoE, "std_swiglu_fp32_E4_d32_F64_M29", 4, 32, 64, 29, 21)
    standard_swiglu(torch, nn, StandardMoE, "std_swiglu_fp32_E8_d128_F256_M70", 8, 128, 256, 70, 22)
    # CPU-runnable SwiGLU config: d=512, 8 experts, top-2, d_ff=2048, Xavier-normal weights
    # from seed 0; 8 tokens and 64 tokens of N(0,1).  Weights are regenerated from the seed.
    standard_swiglu(torch, nn, StandardMoE, "std_swiglu_fp32_E8_d512_F2048_M8", 8, 512, 2048, 8, 0,
                    x_only_seed=1000)
    standard_swiglu(torch, nn, StandardMoE, "std_swiglu_fp32_E8_d512_F2048_M64", 8, 512, 2048, 64, 0,
                    x_only_seed=1001)
    standard_swiglu_lowp(torch, nn, StandardMoE, "std_swiglu_bf16_E8_d512_F1024_M64", 8, 512, 1024, 64, 51, "bf16")
    ultimate_linear("ult_linear_fp32_ws1_E8_d64_M50", ref, 8, 64, 50, 31, 1)
    ultimate_linear("ult_linear_fp32_ws2_E8_d32_M23", ref, 8, 32, 23, 32, 2)
    ultimate_linear("ult_linear_fp32_ws4_E8_d32_M17", ref, 8, 32, 17, 33, 4)
    topk_ties(torch, "topk_ties", 41)
    grads_fixtures(torch, nn, StandardMoE)
    print("fixtures written to", HERE)


def grads_fixtures(torch, nn, StandardMoE):
    standard_grads(torch, nn, StandardMoE, "grad_std_linear_fp32_E8_d48_M41", "linear", 8, 48, 0, 41, 61)
    standard_grads(torch, nn, StandardMoE, "grad_std_swiglu_fp32_E4_d32_F64_M29", "swiglu", 4, 32, 64, 29, 62)
    standard_grads(torch, nn, StandardMoE, "grad_std_swiglu_fp32_E8_d32_F48_M57", "swiglu", 8, 32, 48, 57, 63)


if __name__ == "__main__":
    # python tests/golden/make_golden.py <path of the reference checkout> [grads]
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_golden.py <path of the SwiftMoE reference checkout> [grads]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else None)
