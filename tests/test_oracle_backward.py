"""The oracle's layer backward (``moe_backward``): pinned to gradients of the reference's
own StandardMoE (autograd through its unmodified forward, fp32; the reference itself is
forward-only), and checked against torch autograd of an independent float64
restatement for what the reference lacks (capacity drops, shared expert, router
offsets, pre-weighting, k != 2)."""
import numpy as np
import pytest
import torch

import fixtures as fx
from oracle import moe_oracle as O

pytestmark = pytest.mark.autograd      # the float64 restatement differentiates with torch autograd


def _close(a, b, tol):
    return np.abs(np.asarray(a) - np.asarray(b)).max(initial=0.0) <= tol * max(1.0, np.abs(b).max(initial=0.0))


@pytest.mark.parametrize("name", fx.GRADS)
def test_backward_matches_reference_autograd(name):
    f, p = fx.std_grads(name)
    (out,) = O.moe_forward([f["x"]], p, weighting="post")
    assert _close(out, f["out"], 1e-5)
    g = O.moe_backward(f["x"], p, f["dout"], k=2, weighting="post")
    assert _close(g["x"], f["dx"], 1e-5)
    assert _close(g["gate"], f["dgate"], 1e-5)
    if p.expert_type == "linear":
        assert _close(g["expert_w"].transpose(0, 2, 1), f["dexpert"], 1e-5)   # reference: [out, in]
    else:
        for n in ("w1", "w3", "w2"):
            assert _close(g[n], f["d" + n], 1e-5), n


def _torch_layer(x, p, k, idx, keep, weighting, dout):
    """float64 torch restatement: every expert on every token, gathered per slot."""
    t = lambda a: torch.tensor(np.asarray(a, np.float64), requires_grad=True)
    X, Wg = t(x), t(p.gate)
    logits = X @ Wg.T
    if p.logit_bias is not None:
        logits = logits + torch.tensor(p.logit_bias, dtype=torch.float64)
    w = torch.softmax(logits.gather(1, torch.from_numpy(idx.astype(np.int64))), dim=1)
    w = w * torch.from_numpy(keep.astype(np.float64))          # dropped slots add nothing
    params = {}
    if p.expert_type == "linear":
        params["expert_w"] = t(p.expert_w)
        expert = lambda e, inp: inp @ params["expert_w"][e]
    else:
        for n in ("w1", "w3", "w2"):
            params[n] = t(getattr(p, n))
        expert = lambda e, inp: (torch.nn.functional.silu(inp @ params["w1"][e].T) * (inp @ params["w3"][e].T)
                                 @ params["w2"][e].T)
    rows = torch.arange(x.shape[0])
    out = 0
    for j in range(k):
        e_j = torch.from_numpy(idx[:, j].astype(np.int64))
        wj = w[:, j:j + 1]
        if weighting == "pre":      # the gate weight scales the expert's input
            Y = torch.stack([expert(e, wj * X) for e in range(p.num_experts)])
            out = out + Y[e_j, rows]
        else:                       # ... or its output
            Y = torch.stack([expert(e, X) for e in range(p.num_experts)])
            out = out + wj * Y[e_j, rows]
    if p.sw1 is not None:
        for n in ("sw1", "sw3", "sw2"):
            params[n] = t(getattr(p, n))
        out = out + (torch.nn.functional.silu(X @ params["sw1"][0].T) * (X @ params["sw3"][0].T)) @ params["sw2"][0].T
    (out * torch.from_numpy(np.asarray(dout, np.float64))).sum().backward()
    grads = {n: v.grad.numpy() for n, v in params.items()}
    grads.update(x=X.grad.numpy(), gate=Wg.grad.numpy())
    return grads


@pytest.mark.parametrize("kind,weighting,k,cf,shared,bias", [
    ("linear", "pre", 2, None, False, False), ("linear", "post", 3, 0.6, False, True),
    ("swiglu", "post", 2, 0.8, True, False), ("swiglu", "post", 4, None, True, True)])
def test_backward_matches_float64_autograd(kind, weighting, k, cf, shared, bias):
    rng = np.random.default_rng(k * 7 + int(shared))
    E, d, F, T = 8, 12, 20, 31
    r = lambda *s: (rng.standard_normal(s) * 0.3).astype(np.float32)
    p = O.MoEParams(gate=r(E, d), expert_type=kind)
    if kind == "linear":
        p.expert_w = r(E, d, d)
    else:
        p.w1, p.w3, p.w2 = r(E, F, d), r(E, F, d), r(E, d, F)
    if shared:
        p.sw1, p.sw3, p.sw2 = r(1, F, d), r(1, F, d), r(1, d, F)
    if bias:
        p.logit_bias = (rng.standard_normal(E) * 1.5).astype(np.float32)
    x = rng.standard_normal((T, d)).astype(np.float32)
    dout = rng.standard_normal((T, d)).astype(np.float32)
    _, aux = O.moe_forward([x], p, k=k, capacity_factor=cf, return_aux=True)
    idx = aux["routed"][0][0]
    keep = aux["kept"][0]
    ref = _torch_layer(x, p, k, idx, keep, weighting, dout)
    g = O.moe_backward(x, p, dout, k=k, weighting=weighting, capacity_factor=cf)
    assert set(ref) <= set(g)
    for n, v in ref.items():
        # the oracle's gate weights come from its float32 router, as in its forward
        assert _close(g[n], v, 1e-6), n
