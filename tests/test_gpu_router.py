"""Router kernels (C ABI) against the oracle and the reference's torch.topk outputs."""
import numpy as np
import pytest
import torch

import fixtures as fx
from oracle import moe_oracle as O
from util import max_abs_err, routing_matches_up_to_ties, rounded, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from swiftmoe_b200 import kernels
    return kernels


def test_topk_from_reference_logits_bit_exact(K):
    """Fed the reference's own router logits, indices and per-expert counts are bit-exact."""
    for name in fx.STD_LINEAR + ["std_linear_fp16_E8_d128_M33"]:
        f = fx.load(name)
        lg = f["logits"]
        if lg.shape[0] == 0:
            continue
        idx, w = K.topk_from_logits(to_dev(lg), 2)
        idx = idx.cpu().numpy()
        assert (idx == f["topk_idx"]).all(), name
        E = lg.shape[1]
        assert (np.bincount(idx.ravel(), minlength=E) == np.bincount(f["topk_idx"].ravel(), minlength=E)).all()
        np.testing.assert_allclose(w.cpu().numpy(), f["topk_w"], atol=1e-3 if "fp16" in name else 1e-6)


def test_topk_ties_lower_index(K):
    f = fx.load("topk_ties")
    for c in sorted({k.rsplit("_", 1)[0] for k in f}):
        lg = f[c + "_logits"]
        k = f[c + "_idx"].shape[1]
        idx, w = K.topk_from_logits(to_dev(lg), k)
        v_ref, i_ref = O.topk_lower_index(lg, k)
        assert (idx.cpu().numpy() == i_ref).all(), c            # lower-index rule, bit-exact
        sel = np.take_along_axis(lg, idx.cpu().numpy().astype(np.int64), 1)
        assert (sel == f[c + "_vals"]).all(), c                 # same values as torch.topk
        E = lg.shape[1]
        assert (np.bincount(idx.cpu().numpy().ravel(), minlength=E) ==
                np.bincount(i_ref.ravel(), minlength=E)).all()
        np.testing.assert_allclose(w.cpu().numpy(), f[c + "_w"], atol=2e-6)


def test_topk_nan_and_inf(K):
    lg = np.random.default_rng(1).standard_normal((64, 16)).astype(np.float32)
    lg[3, 7] = np.nan
    lg[5, [2, 9]] = np.nan
    lg[8, 4] = np.inf
    lg[9, :] = -np.inf
    idx, _ = K.topk_from_logits(to_dev(lg), 3)
    _, i_ref = O.topk_lower_index(lg, 3)
    assert (idx.cpu().numpy() == i_ref).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,d,E,k", [(1, 64, 8, 2), (63, 128, 8, 2), (64, 256, 8, 2), (65, 512, 8, 1),
                                     (300, 4096, 8, 2), (257, 96, 7, 3), (100, 128, 16, 4), (77, 64, 32, 8),
                                     (200, 256, 64, 8), (130, 128, 128, 8), (50, 72, 40, 2), (33, 20, 5, 5),
                                     # decode-sized batches (T <= 64, d % 512 == 0): 16 warps per 16 tokens
                                     (1, 4096, 8, 2), (17, 1024, 16, 4), (64, 512, 32, 8), (40, 2048, 24, 3)])
def test_router_fused_vs_oracle(K, dtype, T, d, E, k):
    rng = np.random.default_rng(T * 1000 + E)
    x = rounded(rng.standard_normal((T, d)).astype(np.float32), dtype)
    g = rounded((rng.standard_normal((E, d)) * 0.05).astype(np.float32), dtype)
    bias = (rng.standard_normal(E) * 1.5).astype(np.float32) if E >= 16 else None
    idx, w, logits = K.router(to_dev(x, dtype), to_dev(g, dtype), k,
                              to_dev(bias) if bias is not None else None, return_logits=True)
    lg_ref = O.gate_logits(x, g, None, acc=np.float64)
    scale = np.abs(lg_ref).max()
    assert max_abs_err(logits.cpu().numpy(), lg_ref) <= 1e-5 * max(scale, 1.0) * max(1, d / 512)
    lgb = lg_ref + (bias[None, :] if bias is not None else 0)
    v_ref, i_ref = O.topk_lower_index(lgb.astype(np.float32), k)
    bad = routing_matches_up_to_ties(idx.cpu().numpy(), i_ref, lgb)
    assert not bad, f"rows with non-tie routing differences: {bad[:5]}"
    ok = (idx.cpu().numpy() == i_ref).all(1)
    np.testing.assert_allclose(w.cpu().numpy()[ok], O.softmax_rows(v_ref)[ok], atol=1e-5)


def test_router_empty(K):
    x = torch.empty((0, 64), device="cuda", dtype=torch.bfloat16)
    g = torch.randn((8, 64), device="cuda", dtype=torch.bfloat16)
    idx, w = K.router(x, g, 2)
    assert idx.shape == (0, 2) and w.shape == (0, 2)
