"""Parity at the full benchmark sizes through properties that do not need the whole
oracle run: without a capacity limit every token's output depends only on its own
routing, so a sample of tokens from a full-size forward is checked against a plain
PyTorch fp32 reference of those tokens; dispatch plans at full size are compared with
the oracle's index-order plan bit for bit."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from util import max_rel_err

pytestmark = pytest.mark.gpu


@torch.no_grad()
def _fp32_reference_tokens(x, gate, w1, w3, w2, k, tok, bias=None, shared=None):
    """Layer output of the tokens `tok`, everything in fp32 (torch, on the GPU)."""
    xs = x[tok].float()
    logits = xs @ gate.float().T
    if bias is not None:
        logits = logits + bias.float()
    v, idx = torch.topk(logits, k, dim=-1)
    w = torch.softmax(v, dim=-1)
    out = torch.zeros_like(xs)
    for j in range(k):
        for n in range(xs.shape[0]):
            e = int(idx[n, j])
            h = torch.nn.functional.silu(xs[n] @ w1[e].float().T) * (xs[n] @ w3[e].float().T)
            out[n] += w[n, j] * (h @ w2[e].float().T)
    if shared is not None:
        s1, s3, s2 = (t.float() for t in shared)
        out += (torch.nn.functional.silu(xs @ s1.T) * (xs @ s3.T)) @ s2.T
    return out, idx


def _layer(E, d, F, k, dev, seed, shared=False):
    import swiftmoe_b200 as S
    torch.manual_seed(seed)
    return S.UltimateMoE(E, d, use_fp16=False, dtype=torch.bfloat16, top_k=k, expert_type="swiglu", d_ff=F,
                         num_shared_experts=1 if shared else 0, d_ff_shared=F, use_nccl_opt=False, device=dev)


@pytest.mark.parametrize("T", [16384, 1, 8, 64, 256])
def test_mixtral_shape_token_sample(T):
    """d 4096, 8 experts, top-2, SwiGLU 14336: the bench layer and the decode sweep."""
    dev = torch.device("cuda", 0)
    m = _layer(8, 4096, 14336, 2, dev, seed=0)
    x = torch.randn(T, 4096, device=dev, dtype=torch.bfloat16, generator=torch.Generator(dev).manual_seed(1))
    out = m(x)
    tok = torch.randperm(T, generator=torch.Generator().manual_seed(2))[:24].to(dev)
    ref, ridx = _fp32_reference_tokens(x, m.gate_weight, m.w1, m.w3, m.w2, 2, tok)
    from swiftmoe_b200 import kernels
    idx, _ = kernels.router(x, m.gate_weight, 2)
    same = (torch.sort(idx[tok].long(), 1)[0] == torch.sort(ridx, 1)[0]).all(1).cpu().numpy()
    assert same.mean() > 0.9
    assert max_rel_err(out[tok].float().cpu().numpy()[same], ref.cpu().numpy()[same]) <= 2e-2


def test_fine_grained_shape_token_sample():
    """d 2048, 128 routed experts + 1 shared, top-8, SwiGLU 1024, 32768 tokens, skewed
    router (per-expert logit offsets ~ N(0, 1.5))."""
    dev = torch.device("cuda", 0)
    m = _layer(128, 2048, 1024, 8, dev, seed=3, shared=True)
    bias = torch.randn(128, generator=torch.Generator().manual_seed(2)) * 1.5
    m.set_logit_bias(bias)
    x = torch.randn(32768, 2048, device=dev, dtype=torch.bfloat16, generator=torch.Generator(dev).manual_seed(4))
    out = m(x)
    tok = torch.randperm(32768, generator=torch.Generator().manual_seed(5))[:16].to(dev)
    ref, ridx = _fp32_reference_tokens(x, m.gate_weight, m.w1, m.w3, m.w2, 8, tok, bias=m.logit_bias,
                                       shared=(m.shared_w1, m.shared_w3, m.shared_w2))
    from swiftmoe_b200 import kernels
    idx, _ = kernels.router(x, m.gate_weight, 8, m.logit_bias)
    same = (torch.sort(idx[tok].long(), 1)[0] == torch.sort(ridx, 1)[0]).all(1).cpu().numpy()
    assert same.mean() > 0.8
    assert max_rel_err(out[tok].float().cpu().numpy()[same], ref.cpu().numpy()[same]) <= 2e-2


@pytest.mark.parametrize("T,k,E,cf", [(32768, 8, 128, None), (65536, 2, 64, 1.25)])
def test_full_size_plan_bit_exact(T, k, E, cf):
    """C4 routing shape, and the C3 capacity cut (8 x 8192 tokens, 64 experts, cf 1.25 ->
    2560 rows per expert) with skewed logits so experts overflow."""
    from swiftmoe_b200 import kernels
    from swiftmoe_b200._core import capacity_rows
    g = torch.Generator().manual_seed(T)
    logits = torch.randn(T, E, generator=g) + torch.randn(E, generator=g) * 1.5
    idx, _ = kernels.topk_from_logits(logits.cuda(), k)
    cap = capacity_rows(cf, T, 1, k, E)
    plan = kernels.dispatch_plan(idx, E, cap)
    idx_n = idx.cpu().numpy()
    rows, kept = O.dispatch_plan([idx_n], E, 1, cap if cap > 0 else None)
    kept_n = np.array([len(r) for r in rows])
    offsets = np.concatenate([[0], np.cumsum(kept_n)])
    assert (plan["counts"].cpu().numpy() == np.bincount(idx_n.ravel(), minlength=E)).all()
    assert (plan["offsets"].cpu().numpy() == offsets).all()
    expect = -np.ones(T * k, np.int64)
    for e in range(E):
        r = rows[e]
        expect[r[:, 1] * k + r[:, 2]] = offsets[e] + np.arange(len(r))
    assert (plan["slot_row"].cpu().numpy() == expect).all()
    if cap:
        assert kept_n.max() <= cap and (np.bincount(idx_n.ravel(), minlength=E) > cap).any()
