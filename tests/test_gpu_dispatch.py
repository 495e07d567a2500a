"""Dispatch plan / permute / combine / gather / EP regroup kernels (C ABI), bit-exact
against the oracle's index-order plan."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from util import max_abs_err, rounded, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from swiftmoe_b200 import kernels
    return kernels


def expected_plan(idx: np.ndarray, E: int, capacity: int, row_align: int):
    T, k = idx.shape
    plan, kept = O.dispatch_plan([idx], E, 1, capacity if capacity > 0 else None)
    counts = np.bincount(idx.ravel(), minlength=E)
    kept_n = np.array([len(p) for p in plan])
    aligned = (kept_n + row_align - 1) // row_align * row_align
    offsets = np.concatenate([[0], np.cumsum(aligned)]).astype(np.int64)
    slot_row = -np.ones(T * k, np.int64)
    row_token = {}
    for e in range(E):
        for n, (_, t, j) in enumerate(plan[e]):
            slot_row[t * k + j] = offsets[e] + n
            row_token[offsets[e] + n] = t
        for r in range(offsets[e] + kept_n[e], offsets[e + 1]):
            row_token[r] = -1
    return counts, offsets, slot_row, row_token


@pytest.mark.parametrize("T,k,E,cap,align", [(0, 2, 8, 0, 1), (1, 2, 8, 0, 1), (63, 2, 8, 0, 1), (64, 2, 8, 0, 1),
                                             (65, 2, 8, 0, 128), (1000, 2, 8, 0, 1), (5000, 8, 128, 0, 1),
                                             (3000, 2, 64, 100, 1), (777, 3, 7, 50, 16), (9000, 2, 8, 2000, 1),
                                             (20000, 8, 130, 900, 8),
                                             # one-block plans (T * k <= 2048: one launch)
                                             (600, 3, 7, 50, 16), (256, 8, 128, 0, 1), (1024, 2, 8, 300, 1),
                                             (2048, 1, 3000, 0, 1), (1, 2, 4096, 0, 4), (2049, 1, 8, 0, 1)])
def test_plan_bit_exact(K, T, k, E, cap, align):
    rng = np.random.default_rng(T + E)
    # skewed routing: some experts much more popular
    p = rng.dirichlet(np.ones(E) * 0.3)
    p = (p + 1e-3) / (p + 1e-3).sum()
    idx = np.array([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)], dtype=np.int32).reshape(T, k)
    plan = K.dispatch_plan(to_dev(idx, torch.int32), E, cap, align)
    counts, offsets, slot_row, row_token = expected_plan(idx, E, cap, align)
    assert (plan["counts"].cpu().numpy() == counts).all()
    assert (plan["offsets"].cpu().numpy() == offsets).all()
    assert (plan["slot_row"].cpu().numpy() == slot_row).all()
    rt = plan["row_token"].cpu().numpy()
    for r, t in row_token.items():
        assert rt[r] == t
    assert plan["rows_cap"] >= offsets[-1]


def test_plan_all_to_one_expert(K):
    T, k, E = 4097, 2, 8
    idx = np.zeros((T, k), np.int32)
    idx[:, 1] = 5
    plan = K.dispatch_plan(to_dev(idx, torch.int32), E, 0, 1)
    counts, offsets, slot_row, _ = expected_plan(idx, E, 0, 1)
    assert (plan["offsets"].cpu().numpy() == offsets).all()
    assert (plan["slot_row"].cpu().numpy() == slot_row).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,d,k,E", [(1, 64, 2, 8), (129, 512, 2, 8), (300, 36, 3, 5), (1000, 2048, 8, 64)])
def test_permute_combine(K, dtype, T, d, k, E):
    rng = np.random.default_rng(d + T)
    idx = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    x = rounded(rng.standard_normal((T, d)).astype(np.float32), dtype)
    w = rng.random((T, k)).astype(np.float32)
    cap = max(1, (T * k) // E)  # forces drops
    plan = K.dispatch_plan(to_dev(idx, torch.int32), E, cap, 1)
    rows = K.permute_rows(to_dev(x, dtype), plan["row_token"], plan["offsets"], plan["rows_cap"])
    total = int(plan["offsets"][-1])
    rt = plan["row_token"].cpu().numpy()[:total]
    assert (rows[:total].float().cpu().numpy() == x[rt]).all()        # bit-exact copy
    # combine: y = rows * 2 + 1 (any row function), weighted sum over kept slots
    y = rows.float() * 2 + 1
    y = y.to(dtype)
    shared = rounded(rng.standard_normal((T, d)).astype(np.float32), dtype)
    out = K.combine(y, plan["slot_row"], to_dev(w), T, k, shared=to_dev(shared, dtype))
    sr = plan["slot_row"].cpu().numpy().reshape(T, k)
    yn = y.float().cpu().numpy()
    ref = shared.astype(np.float64).copy()
    for j in range(k):
        m = sr[:, j] >= 0
        ref[m] += w[m, j, None] * yn[sr[m, j]]
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert max_abs_err(out.float().cpu().numpy(), ref) <= tol * max(1.0, np.abs(ref).max())


def test_gather_rows(K):
    rng = np.random.default_rng(3)
    src = rng.standard_normal((50, 24)).astype(np.float32)
    index = rng.integers(-1, 50, size=80).astype(np.int32)
    out = K.gather_rows(to_dev(src), to_dev(index, torch.int32), 80).cpu().numpy()
    ref = np.where(index[:, None] >= 0, src[np.maximum(index, 0)], 0)
    assert (out == ref).all()


@pytest.mark.parametrize("ws,El,cap", [(2, 4, 0), (4, 2, 5), (8, 1, 0), (3, 5, 7)])
def test_ep_regroup_plan(K, ws, El, cap):
    rng = np.random.default_rng(ws * 10 + El)
    rc = rng.integers(0, 9, size=(ws, El)).astype(np.int32)
    n_recv = int(rc.sum())
    rg = K.ep_regroup_plan(to_dev(rc, torch.int32), cap, n_recv)
    # reference: receive rows are (src, le)-major; expert rows are (le, src, i)-major
    seg = []
    for s in range(ws):
        for le in range(El):
            seg += [(s, le, i) for i in range(rc[s, le])]
    kept = [min(int(rc[:, le].sum()), cap) if cap > 0 else int(rc[:, le].sum()) for le in range(El)]
    offsets = np.concatenate([[0], np.cumsum(kept)])
    recv_dst = []
    for (s, le, i) in seg:
        pos = int(rc[:s, le].sum()) + i
        recv_dst.append(-1 if (cap > 0 and pos >= cap) else offsets[le] + pos)
    assert (rg["counts"].cpu().numpy() == rc.sum(0)).all()
    assert (rg["offsets"].cpu().numpy() == offsets).all()
    got = rg["recv_dst"].cpu().numpy()[:n_recv]
    assert (got == np.array(recv_dst, dtype=np.int64)).all()
    rs = rg["row_src"].cpu().numpy()
    for r, dst in enumerate(recv_dst):
        if dst >= 0:
            assert rs[dst] == r


@pytest.mark.parametrize("ws,El,cap,chunks", [(2, 4, 9, 3), (4, 2, 5, 2), (8, 1, 40, 4)])
def test_ep_regroup_plan_chunked_capacity(K, ws, El, cap, chunks):
    """Chunk c of a batch exchanged in token chunks: the capacity cut uses each segment's
    position in the whole batch's (source rank, token, slot) order (pos_base)."""
    import ep_doubles
    from swiftmoe_b200.ep import capacity_positions
    rng = np.random.default_rng(ws * 100 + El)
    rc_all = rng.integers(0, 7, size=(chunks, ws, El)).astype(np.int32)
    pos = capacity_positions(rc_all, cap)
    for c in range(chunks):
        rc = rc_all[c]
        n_recv = int(rc.sum())
        got = K.ep_regroup_plan(to_dev(rc, torch.int32), cap, n_recv, pos_base=to_dev(pos[c], torch.int32))
        exp = ep_doubles.ep_regroup_plan(torch.from_numpy(rc), cap, n_recv, torch.from_numpy(pos[c]))
        assert (got["offsets"].cpu().numpy() == exp["offsets"].numpy()).all()
        assert (got["recv_dst"].cpu().numpy()[:n_recv] == exp["recv_dst"].numpy()[:n_recv]).all()
    # the chunks together keep exactly min(total, cap) rows of every expert
    kept = sum(int(K.ep_regroup_plan(to_dev(rc_all[c], torch.int32), cap, int(rc_all[c].sum()),
                                     pos_base=to_dev(pos[c], torch.int32))["offsets"][-1]) for c in range(chunks))
    assert kept == int(np.minimum(rc_all.sum((0, 1)), cap).sum())


def _doubles():
    import ep_doubles
    return ep_doubles


@pytest.mark.parametrize("T,k,E", [(1, 2, 8), (777, 4, 16), (5000, 8, 128)])
def test_plan_skips_minus_one(K, T, k, E):
    """idx entries of -1 are skipped slots: slot_row -1, not counted, no device error."""
    rng = np.random.default_rng(T)
    idx = np.array([rng.choice(E, size=k, replace=False) for _ in range(T)], dtype=np.int32).reshape(T, k)
    idx[rng.random((T, k)) < 0.3] = -1
    plan = K.dispatch_plan(to_dev(idx, torch.int32), E, 0, 1)
    ref = _doubles().dispatch_plan(torch.from_numpy(idx), E)
    for key in ("counts", "offsets", "slot_row"):
        assert (plan[key].cpu().numpy() == ref[key].numpy()).all(), key
    n = int(ref["offsets"][-1])
    assert (plan["row_token"].cpu().numpy()[:n] == ref["row_token"].numpy()[:n]).all()
    assert K.read_device_error("cuda") == 0


@pytest.mark.parametrize("T,k,El,ws,me", [(1, 2, 4, 2, 1), (300, 4, 8, 2, 0), (2000, 8, 16, 8, 3), (999, 6, 2, 4, 2)])
def test_ep_dedup_plan_and_meta(K, T, k, El, ws, me):
    """Token dedup: rotated ranks, the rank plan and the per-row slot metadata, bit-exact
    against the numpy restatement."""
    D = _doubles()
    E = El * ws
    rng = np.random.default_rng(T + k)
    idx = np.array([rng.choice(E, size=k, replace=False) for _ in range(T)], dtype=np.int32).reshape(T, k)
    w = rng.random((T, k)).astype(np.float32)
    ridx = K.ep_dedup_ranks(to_dev(idx, torch.int32), El, ws, me)
    ridx_ref = D.ep_dedup_ranks(torch.from_numpy(idx), El, ws, me)
    assert (ridx.cpu().numpy() == ridx_ref.numpy()).all()
    plan = K.dispatch_plan(ridx, ws, 0, 1)
    me_, mw, oe = K.ep_dedup_meta(to_dev(idx, torch.int32), to_dev(w, torch.float32), ridx, plan["slot_row"],
                                  plan["counts"][0:1], El, ws, plan["rows_cap"])
    ref_plan = D.dispatch_plan(ridx_ref, ws)
    me_r, mw_r, oe_r = D.ep_dedup_meta(torch.from_numpy(idx), torch.from_numpy(w), ridx_ref, ref_plan["slot_row"],
                                       ref_plan["counts"][0:1], El, ws, plan["rows_cap"])
    n = int(ref_plan["offsets"][-1])
    assert (me_.cpu().numpy()[:n] == me_r.numpy()[:n]).all()
    assert (mw.cpu().numpy()[:n] == mw_r.numpy()[:n]).all()
    assert (oe.cpu().numpy()[:T] == oe_r.numpy()[:T]).all()
    assert K.read_device_error("cuda") == 0


@pytest.mark.parametrize("ws,E,cap,seed", [(2, 8, 0, 0), (4, 16, 37, 1), (8, 8, 500, 2), (8, 64, 0, 3), (4, 8, 1, 4)])
def test_ep_layout_matches_restatement(ws, E, cap, seed):
    """Device layout of the exchange (send addresses, kept prefixes, receive offsets,
    return table) from a count matrix, bit for bit against its numpy restatement.  The
    buffer bases are synthetic: the kernel only computes addresses from them."""
    import ep_doubles
    from swiftmoe_b200 import kernels as K
    rng = np.random.default_rng(seed)
    G = rng.integers(0, 300, size=(ws, E)).astype(np.int32)
    G[rng.random((ws, E)) < 0.2] = 0                      # empty segments
    rb = 8192
    bases = [(np.arange(ws, dtype=np.int64) + 1) << 34, (np.arange(ws, dtype=np.int64) + 17) << 34]
    El = E // ws
    for me in range(ws):
        outs = []
        for mod, dev in ((K, "cuda"), (ep_doubles, "cpu")):
            lay = dict(send_addr=torch.zeros(E, dtype=torch.int64, device=dev),
                       keep=torch.zeros(E, dtype=torch.int32, device=dev),
                       recv_offsets=torch.zeros(El + 1, dtype=torch.int32, device=dev),
                       seg=torch.zeros(2 * El * ws + 1, dtype=torch.int64, device=dev))
            mod.ep_layout(torch.from_numpy(G).to(dev), me, cap, torch.from_numpy(bases[0]).to(dev),
                          torch.from_numpy(bases[1]).to(dev), rb, 10 ** 6, lay)
            outs.append({k_: v.cpu().numpy() for k_, v in lay.items()})
        for key in outs[0]:
            assert (outs[0][key] == outs[1][key]).all(), (me, key)


def test_ep_layout_overflow_guard():
    """A receive buffer that would overflow: nothing is addressed, and the error word says so."""
    from swiftmoe_b200 import kernels as K
    G = torch.full((2, 4), 100, dtype=torch.int32, device="cuda")
    base = torch.tensor([1 << 34, 2 << 34], dtype=torch.int64, device="cuda")
    lay = dict(send_addr=torch.ones(4, dtype=torch.int64, device="cuda"), keep=torch.ones(4, dtype=torch.int32, device="cuda"),
               recv_offsets=torch.ones(3, dtype=torch.int32, device="cuda"),
               seg=torch.ones(9, dtype=torch.int64, device="cuda"))
    K.read_device_error(torch.device("cuda", 0))
    K.ep_layout(G, 0, 0, base, base, 4096, 150, lay)      # each rank would receive 200 rows
    assert int(lay["send_addr"].abs().sum()) == 0 and int(lay["keep"].sum()) == 0
    assert int(lay["recv_offsets"].sum()) == 0
    assert K.read_device_error(torch.device("cuda", 0)) == 4


@pytest.mark.parametrize("cap", [0, 40])
def test_ep_send_rows_and_drop_slots(cap):
    """The send kernel stores each routed row of the other ranks' experts at its place in
    the owner's expert-major receive buffer (here: local buffers standing in for the
    peers'), rows past the capacity cut are not sent, and drop_slots marks exactly the
    cut slots -- against the numpy restatement."""
    import ep_doubles
    from swiftmoe_b200 import kernels as K
    ws, E, T, k, d, me = 4, 8, 300, 2, 256, 1
    El = E // ws
    rng = np.random.default_rng(11)
    idx = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    x = torch.randn(T, d, device="cuda").to(torch.bfloat16)
    plan = K.dispatch_plan(torch.from_numpy(idx).cuda(), E)
    # every rank's counts: this rank's from the plan, the others' random
    G = rng.integers(0, 160, size=(ws, E)).astype(np.int32)
    G[me] = plan["counts"].cpu().numpy()
    rb = d * 2
    rows_max = ws * T * k
    bufs = [torch.zeros(rows_max, d, dtype=torch.bfloat16, device="cuda") for _ in range(ws)]
    base = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    lay = dict(send_addr=torch.zeros(E, dtype=torch.int64, device="cuda"),
               keep=torch.zeros(E, dtype=torch.int32, device="cuda"),
               recv_offsets=torch.zeros(El + 1, dtype=torch.int32, device="cuda"),
               seg=torch.zeros(2 * El * ws + 1, dtype=torch.int64, device="cuda"))
    K.ep_layout(torch.from_numpy(G).cuda(), me, cap, base, base, rb, rows_max, lay)
    K.ep_send_rows(x, plan["row_token"], plan["offsets"], me * El, El, lay["send_addr"], lay["keep"],
                   plan["rows_cap"])
    torch.cuda.synchronize()
    # restatement on the host: the same layout, rows copied into host copies of the buffers
    hb = [torch.zeros(rows_max, d, dtype=torch.bfloat16) for _ in range(ws)]
    hbase = torch.tensor([b.data_ptr() for b in hb], dtype=torch.int64)
    hl = dict(send_addr=torch.zeros(E, dtype=torch.int64), keep=torch.zeros(E, dtype=torch.int32),
              recv_offsets=torch.zeros(El + 1, dtype=torch.int32), seg=torch.zeros(2 * El * ws + 1, dtype=torch.int64))
    ep_doubles.ep_layout(torch.from_numpy(G), me, cap, hbase, hbase, rb, rows_max, hl)
    ep_doubles.ep_send_rows(x.cpu(), plan["row_token"].cpu(), plan["offsets"].cpu(), me * El, El,
                            hl["send_addr"], hl["keep"], plan["rows_cap"])
    for r in range(ws):
        assert torch.equal(bufs[r].cpu(), hb[r]), r
    sr = plan["slot_row"].clone()
    K.ep_drop_slots(torch.from_numpy(idx).cuda(), plan["offsets"], lay["keep"], sr)
    sr_h = plan["slot_row"].cpu().clone()
    ep_doubles.ep_drop_slots(torch.from_numpy(idx), plan["offsets"].cpu(), hl["keep"], sr_h)
    assert torch.equal(sr.cpu(), sr_h)
    assert (sr.cpu() < 0).any() == (cap > 0 and bool((G[:me + 1].sum(0) > cap).any()))


@pytest.mark.parametrize("ws,seed", [(2, 5), (4, 6), (8, 7)])
def test_ep_layout_rotated_matches_restatement(ws, seed):
    """The token-dedup layout: every source's groups in its own rotated rank order."""
    import ep_doubles
    from swiftmoe_b200 import kernels as K
    rng = np.random.default_rng(seed)
    G = rng.integers(0, 500, size=(ws, ws)).astype(np.int32)
    bases = [(np.arange(ws, dtype=np.int64) + 3) << 34, (np.arange(ws, dtype=np.int64) + 29) << 34]
    for me in range(ws):
        outs = []
        for mod, dev in ((K, "cuda"), (ep_doubles, "cpu")):
            lay = dict(send_addr=torch.zeros(ws, dtype=torch.int64, device=dev),
                       keep=torch.zeros(ws, dtype=torch.int32, device=dev),
                       recv_offsets=torch.zeros(2, dtype=torch.int32, device=dev),
                       seg=torch.zeros(2 * ws + 1, dtype=torch.int64, device=dev))
            mod.ep_layout(torch.from_numpy(G).to(dev), me, 0, torch.from_numpy(bases[0]).to(dev),
                          torch.from_numpy(bases[1]).to(dev), 4096, 10 ** 6, lay, rotated=True)
            outs.append({k_: v.cpu().numpy() for k_, v in lay.items()})
        for key in outs[0]:
            assert (outs[0][key] == outs[1][key]).all(), (me, key)


def test_clear_tail_store_rows_copy_rows_count():
    """The dedup schedule's small kernels: unfilled receive rows marked -1, rows stored at
    per-row addresses (0 = skipped), and a copy of a device-counted prefix of rows."""
    from swiftmoe_b200 import kernels as K
    idx = torch.arange(40, dtype=torch.int32, device="cuda").view(10, 4)
    K.ep_clear_tail(idx, torch.tensor([6], dtype=torch.int32, device="cuda"))
    assert (idx[:6].cpu() == torch.arange(24, dtype=torch.int32).view(6, 4)).all() and (idx[6:] == -1).all()
    src = torch.randn(9, 64, device="cuda").to(torch.bfloat16)
    dst = torch.zeros(20, 64, device="cuda", dtype=torch.bfloat16)
    order = [4, 0, 17, 9, -1, 3, 12, 19, 7]          # -1: row not stored
    ptrs = torch.tensor([0 if o < 0 else dst[o].data_ptr() for o in order], dtype=torch.int64, device="cuda")
    K.store_rows(src, ptrs, 9)
    torch.cuda.synchronize()
    for r, o in enumerate(order):
        if o >= 0:
            assert torch.equal(dst[o], src[r])
    assert int((dst.float().abs().sum(1) > 0).sum()) == 8
    out = torch.zeros(9, 64, device="cuda", dtype=torch.bfloat16)
    K.copy_rows_count(out, src, torch.tensor([5], dtype=torch.int32, device="cuda"))
    assert torch.equal(out[:5], src[:5]) and (out[5:] == 0).all()
