"""Layer backward on one GPU (16-bit SwiGLU layers): the K-grouped weight-gradient GEMM
and the gate/up epilogue against float32 torch matmuls, and the gradients of the whole
layer -- x, the gate and every expert weight, with capacity drops, a shared expert and
router offsets -- against the oracle's moe_backward (float64, on the same bf16-rounded
inputs and the GPU's own routing), which is pinned to the reference's autograd
gradients.  Tolerance (bf16): max|grad - ref| / max|ref| <= 2e-2 per gradient."""
import numpy as np
import pytest
import torch

import synth
from oracle import moe_oracle as O
from util import max_rel_err, rounded

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from swiftmoe_b200 import kernels
    return kernels


@pytest.mark.parametrize("koff,M,N,K_,ld", [
    ([0, 128, 128, 320], 200, 264, 320, 320),     # an empty group in the middle, ragged M and N
    ([0, 64, 448], 384, 512, 448, 456),           # row stride larger than K
    ([0, 300], 256, 256, 300, 304)])              # one group ending off a 64-row boundary (K tail reads zeros)
def test_wgrad_gemm_matches_torch(K, koff, M, N, K_, ld):
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, ld, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, ld, device="cuda", generator=g).to(torch.bfloat16)
    ko = torch.tensor(koff, dtype=torch.int32, device="cuda")
    C = K.wgrad_gemm(A, B, ko, K=K_)
    for i in range(len(koff) - 1):
        a, b = koff[i], koff[i + 1]
        ref = A[:, a:b].float() @ B[:, a:b].float().T
        if b == a:
            assert (C[i] == 0).all()
        else:
            assert (C[i] - ref).abs().max().item() <= 1e-4 * max(ref.abs().max().item(), 1.0)
    assert K.read_device_error(torch.device("cuda", 0)) == 0


@pytest.mark.parametrize("koff,M,N,K_,lda,ldb", [
    ([0, 128, 128, 320], 200, 264, 320, 200, 264),   # an empty group, ragged M and N
    ([0, 64, 448], 384, 512, 448, 392, 520),          # row strides wider than M / N
    ([0, 300], 256, 256, 300, 256, 256),              # one group ending off a 64-row boundary (rows past K read zeros)
    ([0, 4096, 8192], 1024, 512, 8192, 1024, 512)])   # long K ranges
def test_wgrad_gemm_rows_matches_torch(K, koff, M, N, K_, lda, ldb):
    """The weight-gradient GEMM on operands given as rows of K (the routed rows as they
    are, read as MN-major tensor-core tiles): C[g] = A[K_g, :M]^T B[K_g, :N]."""
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randn(K_ + 5, lda, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(K_ + 5, ldb, device="cuda", generator=g).to(torch.bfloat16)
    ko = torch.tensor(koff, dtype=torch.int32, device="cuda")
    C = K.wgrad_gemm_rows(A[:K_].contiguous(), B[:K_].contiguous(), ko, M=M, N=N)
    for i in range(len(koff) - 1):
        a, b = koff[i], koff[i + 1]
        ref = A[a:b, :M].float().T @ B[a:b, :N].float()
        if b == a:
            assert (C[i] == 0).all()
        else:
            assert (C[i] - ref).abs().max().item() <= 1e-4 * max(ref.abs().max().item(), 1.0), i
    assert K.read_device_error(torch.device("cuda", 0)) == 0


def test_gateup_epilogue_matches_torch(K):
    from swiftmoe_b200 import _lib as L
    g = torch.Generator(device="cuda").manual_seed(6)
    rows, d, F = 390, 256, 384
    A = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16)
    W1 = (torch.randn(3, F, d, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    W3 = (torch.randn(3, F, d, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    offs = torch.tensor([0, 130, 131, 390], dtype=torch.int32, device="cuda")
    out = torch.empty(rows, 2 * F, dtype=torch.bfloat16, device="cuda")
    L.check(L.load().smoe_grouped_gemm(L.ptr(A), L.ptr(W1), L.ptr(W3), L.ptr(out), L.SMOE_BF16, L.SMOE_BF16,
                                       L.SMOE_EPI_GATEUP, L.ptr(offs), None, 3, rows, F, d,
                                       L.stream_handle(A.device)), "gateup")
    for e in range(3):
        a, b = int(offs[e]), int(offs[e + 1])
        ga = A[a:b].float() @ W1[e].float().T
        up = A[a:b].float() @ W3[e].float().T
        assert max_rel_err(out[a:b, :F].float().cpu().numpy(), ga.cpu().numpy()) <= 1e-2
        assert max_rel_err(out[a:b, F:].float().cpu().numpy(), up.cpu().numpy()) <= 1e-2


# (T, d, E, k, F, capacity factor, shared expert, router offset std)
LAYERS = [(300, 256, 8, 2, 512, None, False, 0.0),
          (257, 128, 16, 4, 256, 0.6, True, 1.5),
          (64, 256, 8, 2, 256, None, True, 0.0)]


def _layer(T, d, E, k, F, cf, shared, bias_std, seed=0):
    import swiftmoe_b200 as S
    dt = torch.bfloat16
    w1, w3, w2 = synth.swiglu_weights(seed + 3, E, d, F, init="normal", std=0.05)
    gw = synth.normal(seed + 4, (E, d), 0.1)
    sw = synth.swiglu_weights(seed + 5, 1, d, F, init="normal", std=0.05) if shared else None
    bias = synth.normal(seed + 6, (E,), bias_std) if bias_std else None
    m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, expert_type="swiglu", d_ff=F,
                      capacity_factor=cf, num_shared_experts=1 if shared else 0, d_ff_shared=F,
                      use_nccl_opt=False, device=torch.device("cuda", 0))
    with torch.no_grad():
        m.gate_weight.copy_(torch.from_numpy(gw))
        m.w1.copy_(torch.from_numpy(w1)); m.w3.copy_(torch.from_numpy(w3)); m.w2.copy_(torch.from_numpy(w2))
        if shared:
            m.shared_w1.copy_(torch.from_numpy(sw[0][0])); m.shared_w3.copy_(torch.from_numpy(sw[1][0]))
            m.shared_w2.copy_(torch.from_numpy(sw[2][0]))
    if bias is not None:
        m.set_logit_bias(torch.from_numpy(bias))
    r = lambda a: rounded(a, dt)
    p = O.MoEParams(gate=r(gw), expert_type="swiglu", w1=r(w1), w3=r(w3), w2=r(w2))
    p.logit_bias = bias
    if shared:
        p.sw1, p.sw3, p.sw2 = r(sw[0]), r(sw[1]), r(sw[2])
    x = r(synth.normal(seed + 100, (T, d), 1.0))
    dout = r(synth.normal(seed + 200, (T, d), 1.0))
    return m, p, x, dout


@pytest.mark.autograd
@pytest.mark.parametrize("cfg", LAYERS)
def test_layer_backward_matches_oracle(K, cfg):
    T, d, E, k, F, cf, shared, bias_std = cfg
    m, p, x, dout = _layer(*cfg)
    xt = torch.from_numpy(x).to("cuda", torch.bfloat16).requires_grad_(True)
    out = m(xt)
    assert out.requires_grad
    out.backward(torch.from_numpy(dout).to("cuda", torch.bfloat16))
    idx, w = K.router(xt.detach(), m.gate_weight.detach(), k, m.logit_bias)
    ref = O.moe_backward(x, p, dout, k=k, capacity_factor=cf, routing=(idx.cpu().numpy(), w.cpu().numpy()))
    got = {"x": xt.grad, "gate": m.gate_weight.grad, "w1": m.w1.grad, "w3": m.w3.grad, "w2": m.w2.grad}
    if shared:
        got.update(sw1=m.shared_w1.grad, sw3=m.shared_w3.grad, sw2=m.shared_w2.grad)
    for n, v in got.items():
        g_ref = ref[n] if n not in ("sw1", "sw3", "sw2") else ref[n][0]
        err = max_rel_err(v.float().cpu().numpy(), g_ref)
        assert err <= 2e-2, (n, err)
    assert K.read_device_error(torch.device("cuda", 0)) == 0


@pytest.mark.autograd
def test_standard_moe_gradients_reach_each_expert(K):
    """StandardMoE's experts are separate nn.Linear modules: the layer's gradient lands on
    each of them, equal to UltimateMoE's stacked gradient for the same weights."""
    import swiftmoe_b200 as S
    m, p, x, dout = _layer(*LAYERS[0])
    s = S.StandardMoE(8, 256, use_fp16=False, dtype=torch.bfloat16, expert_type="swiglu", d_ff=512).cuda()
    with torch.no_grad():
        s.gate.weight.copy_(m.gate_weight)
        for i in range(8):
            s.experts[i].w1.weight.copy_(m.w1[i]); s.experts[i].w3.weight.copy_(m.w3[i])
            s.experts[i].w2.weight.copy_(m.w2[i])
    xt = torch.from_numpy(x).to("cuda", torch.bfloat16)
    do = torch.from_numpy(dout).to("cuda", torch.bfloat16)
    m(xt).backward(do)
    s(xt).backward(do)
    torch.testing.assert_close(s.gate.weight.grad, m.gate_weight.grad, rtol=0, atol=0)
    for i in range(8):
        torch.testing.assert_close(s.experts[i].w1.weight.grad, m.w1.grad[i], rtol=0, atol=0)
        torch.testing.assert_close(s.experts[i].w2.weight.grad, m.w2.grad[i], rtol=0, atol=0)


@pytest.mark.autograd
@pytest.mark.parametrize("cls,T,d,E,k,cf", [("UltimateMoE", 300, 256, 8, 2, None), ("StandardMoE", 257, 128, 16, 2, 0.5),
                                            ("UltimateMoE", 100, 128, 8, 3, None)])
def test_linear_layer_backward_matches_oracle(K, cls, T, d, E, k, cf):
    """The reference's own expert type (a bias-free d x d linear): UltimateMoE's x @ W
    parameter and StandardMoE's per-expert nn.Linear weights, against moe_backward."""
    import swiftmoe_b200 as S
    dt = torch.bfloat16
    W = synth.normal(7, (E, d, d), 0.05)                 # x @ W layout [d_in, d_out]
    gw = synth.normal(8, (E, d), 0.1)
    x = rounded(synth.normal(9, (T, d), 1.0), dt)
    dout = rounded(synth.normal(10, (T, d), 1.0), dt)
    if cls == "UltimateMoE":
        m = S.UltimateMoE(E, d, use_fp16=False, dtype=dt, top_k=k, capacity_factor=cf).cuda()
        with torch.no_grad():
            m.gate_weight.copy_(torch.from_numpy(gw)); m.expert_weights.copy_(torch.from_numpy(W))
        gate_p = m.gate_weight
    else:
        m = S.StandardMoE(E, d, use_fp16=False, dtype=dt, top_k=k, capacity_factor=cf).cuda()
        with torch.no_grad():
            m.gate.weight.copy_(torch.from_numpy(gw))
            for i in range(E):
                m.experts[i].weight.copy_(torch.from_numpy(W[i].T.copy()))
        gate_p = m.gate.weight
    xt = torch.from_numpy(x).to("cuda", dt).requires_grad_(True)
    m(xt).backward(torch.from_numpy(dout).to("cuda", dt))
    idx, w = K.router(xt.detach(), gate_p.detach(), k)
    p = O.MoEParams(gate=rounded(gw, dt), expert_type="linear", expert_w=rounded(W, dt))
    ref = O.moe_backward(x, p, dout, k=k, capacity_factor=cf, routing=(idx.cpu().numpy(), w.cpu().numpy()))
    if cls == "UltimateMoE":
        dW = m.expert_weights.grad.float().cpu().numpy()
    else:
        dW = np.stack([m.experts[i].weight.grad.float().cpu().numpy().T for i in range(E)])
    assert max_rel_err(xt.grad.float().cpu().numpy(), ref["x"]) <= 2e-2
    assert max_rel_err(gate_p.grad.float().cpu().numpy(), ref["gate"]) <= 2e-2
    assert max_rel_err(dW, ref["expert_w"]) <= 2e-2
    assert K.read_device_error(torch.device("cuda", 0)) == 0


@pytest.mark.autograd
def test_backward_outside_its_scope_raises():
    """Layers the backward does not cover (fp32) fail loudly in backward, not with wrong grads."""
    import swiftmoe_b200 as S
    m = S.UltimateMoE(8, 64, use_fp16=False, expert_type="swiglu", d_ff=128).cuda()      # fp32
    out = m(torch.randn(16, 64, device="cuda"))
    with pytest.raises(NotImplementedError):
        out.sum().backward()
