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
def _fp32_reference_tokens(x, gate, w1, w3, w2, idx, tok, bias=None, shared=None):
    """Layer output of the tokens `tok` in fp32 (torch matmuls on the GPU) on the routing
    `idx` the layer chose (weights: softmax of the fp32 logits of those experts), and the
    fp32 router's own top-k for the routing check."""
    xs = x[tok].float()
    logits = xs @ gate.float().T
    if bias is not None:
        logits = logits + bias.float()
    k = idx.shape[1]
    sel = idx[tok].long()
    w = torch.softmax(logits.gather(1, sel), dim=-1)
    out = torch.zeros_like(xs)
    for e in torch.unique(sel).tolist():
        rows, slots = torch.nonzero(sel == e, as_tuple=True)
        h = torch.nn.functional.silu(xs[rows] @ w1[e].float().T) * (xs[rows] @ w3[e].float().T)
        out.index_add_(0, rows, (h @ w2[e].float().T) * w[rows, slots].view(-1, 1))
    if shared is not None:
        s1, s3, s2 = (t.float() for t in shared)
        out += (torch.nn.functional.silu(xs @ s1.T) * (xs @ s3.T)) @ s2.T
    return out, torch.topk(logits, k, dim=-1).indices, logits


def _check_routing(idx_tok, ridx, logits, rtol=1e-4):
    """Rows whose expert sets differ from the fp32 top-k must be near-ties of the fp32 logits."""
    a = torch.sort(idx_tok.long(), 1)[0]
    b = torch.sort(ridx, 1)[0]
    for n in torch.nonzero((a != b).any(1)).flatten().tolist():
        va = torch.sort(logits[n, a[n]])[0]
        vb = torch.sort(logits[n, b[n]])[0]
        assert (va - vb).abs().max().item() <= rtol * logits[n].abs().max().item(), n


def _layer(E, d, F, k, dev, seed, shared=False):
    import swiftmoe_b200 as S
    torch.manual_seed(seed)
    return S.UltimateMoE(E, d, use_fp16=False, dtype=torch.bfloat16, top_k=k, expert_type="swiglu", d_ff=F,
                         num_shared_experts=1 if shared else 0, d_ff_shared=F, use_nccl_opt=False, device=dev)


@pytest.mark.parametrize("T", [16384, 1, 8, 64, 256])
def test_mixtral_shape_token_sample(T):
    """d 4096, 8 experts, top-2, SwiGLU 14336: the bench layer and the decode sweep; every
    sampled token is compared (on the layer's own routing), and the routing itself must
    match the fp32 top-k except at near-ties."""
    dev = torch.device("cuda", 0)
    m = _layer(8, 4096, 14336, 2, dev, seed=0)
    x = torch.randn(T, 4096, device=dev, dtype=torch.bfloat16, generator=torch.Generator(dev).manual_seed(1))
    out = m(x)
    tok = torch.randperm(T, generator=torch.Generator().manual_seed(2))[:64].to(dev)
    from swiftmoe_b200 import kernels
    idx, _ = kernels.router(x, m.gate_weight, 2)
    ref, ridx, logits = _fp32_reference_tokens(x, m.gate_weight, m.w1, m.w3, m.w2, idx, tok)
    _check_routing(idx[tok], ridx, logits)
    assert max_rel_err(out[tok].float().cpu().numpy(), ref.cpu().numpy()) <= 2e-2


def test_fine_grained_shape_token_sample():
    """d 2048, 128 routed experts + 1 shared, top-8, SwiGLU 1024, 32768 tokens, skewed
    router (per-expert logit offsets ~ N(0, 1.5))."""
    dev = torch.device("cuda", 0)
    m = _layer(128, 2048, 1024, 8, dev, seed=3, shared=True)
    bias = torch.randn(128, generator=torch.Generator().manual_seed(2)) * 1.5
    m.set_logit_bias(bias)
    x = torch.randn(32768, 2048, device=dev, dtype=torch.bfloat16, generator=torch.Generator(dev).manual_seed(4))
    out = m(x)
    tok = torch.randperm(32768, generator=torch.Generator().manual_seed(5))[:64].to(dev)
    from swiftmoe_b200 import kernels
    idx, _ = kernels.router(x, m.gate_weight, 8, m.logit_bias)
    ref, ridx, logits = _fp32_reference_tokens(x, m.gate_weight, m.w1, m.w3, m.w2, idx, tok, bias=m.logit_bias,
                                               shared=(m.shared_w1, m.shared_w3, m.shared_w2))
    _check_routing(idx[tok], ridx, logits)
    assert max_rel_err(out[tok].float().cpu().numpy(), ref.cpu().numpy()) <= 2e-2


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


@torch.no_grad()
def test_fp32_layer_token_sample():
    """The fp32 layer (d 512, 8 experts, top-2, SwiGLU 2048, 4096 tokens; the reference's
    use_fp16=False path), whose expert GEMMs run as split tf32 products on the tensor
    cores: 64 sampled tokens against float64 on the layer's own routing, within the fp32
    bar of 1e-5 x the output scale."""
    import swiftmoe_b200 as S
    from swiftmoe_b200 import kernels
    dev = torch.device("cuda", 0)
    torch.manual_seed(5)
    m = S.UltimateMoE(8, 512, use_fp16=False, dtype=torch.float32, top_k=2, expert_type="swiglu", d_ff=2048,
                      use_nccl_opt=False, device=dev)
    x = torch.randn(4096, 512, device=dev, generator=torch.Generator(dev).manual_seed(6))
    out = m(x)
    idx, _ = kernels.router(x, m.gate_weight, 2)
    tok = torch.randperm(4096, generator=torch.Generator().manual_seed(7))[:64].to(dev)
    xs = x[tok].double()
    sel = idx[tok].long()
    w = torch.softmax((xs @ m.gate_weight.double().T).gather(1, sel), dim=-1)
    ref = torch.zeros_like(xs)
    for e in torch.unique(sel).tolist():
        rows, slots = torch.nonzero(sel == e, as_tuple=True)
        h = torch.nn.functional.silu(xs[rows] @ m.w1[e].double().T) * (xs[rows] @ m.w3[e].double().T)
        ref.index_add_(0, rows, (h @ m.w2[e].double().T) * w[rows, slots].view(-1, 1))
    err = (out[tok].double() - ref).abs().max().item()
    assert err <= 1e-5 * max(1.0, ref.abs().max().item()), err
