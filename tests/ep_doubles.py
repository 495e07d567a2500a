"""CPU test double of the swiftmoe_b200.kernels operations used by the expert-parallel
exchange, so that its collective choreography runs on gloo ranks without a GPU.
Each function follows the contract of the C-ABI entry point of the same name."""
import ctypes

import numpy as np
import torch


def dispatch_plan(idx, num_experts, capacity=0, row_align=1):
    idx_n = idx.numpy()
    T, k = idx_n.shape
    E = num_experts
    flat = idx_n.ravel()
    counts = np.bincount(flat[flat >= 0], minlength=E).astype(np.int32)   # -1: skipped slot
    kept = np.minimum(counts, capacity) if capacity > 0 else counts
    aligned = (kept + row_align - 1) // row_align * row_align     # padding rows carry token -1
    offsets = np.concatenate([[0], np.cumsum(aligned)]).astype(np.int32)
    slot_row = -np.ones(T * k, np.int32)
    row_token = -np.ones(max(int(offsets[-1]), 1), np.int32)
    seen = np.zeros(E, np.int64)
    for s in range(T * k):
        e = flat[s]
        if e < 0:
            continue
        if capacity <= 0 or seen[e] < capacity:
            r = offsets[e] + seen[e]
            slot_row[s] = r
            row_token[r] = s // k
        seen[e] += 1
    return dict(counts=torch.from_numpy(counts), offsets=torch.from_numpy(offsets),
                slot_row=torch.from_numpy(slot_row), row_token=torch.from_numpy(row_token),
                rows_cap=int(max(offsets[-1], 1)))


def permute_rows(x, row_token, offsets, rows_cap, out=None):
    first, total = int(offsets[0]), int(offsets[-1])
    rt = row_token.numpy()[first:total]
    xr = x.numpy()
    rows = np.zeros((max(rows_cap, 1), x.shape[1]), xr.dtype) if out is None else out.numpy()
    rows[first:total] = np.where(rt[:, None] >= 0, xr[np.maximum(rt, 0)], 0)
    return torch.from_numpy(rows) if out is None else out


def gather_rows(src, index, n_rows, out=None):
    ind = index.numpy()[:n_rows]
    s = src.numpy()
    o = np.zeros((max(n_rows, 1), src.shape[1]), s.dtype)
    o[:n_rows] = np.where(ind[:, None] >= 0, s[np.maximum(ind, 0)], 0)
    return torch.from_numpy(o)


def ep_regroup_plan(recv_counts, capacity, n_recv, pos_base=None):
    rc = recv_counts.numpy()
    ws, El = rc.shape
    tot = rc.sum(0)
    base = pos_base.numpy() if pos_base is not None else (np.cumsum(rc, 0) - rc)
    kept_seg = np.clip(capacity - base, 0, rc) if capacity > 0 else rc
    kept = kept_seg.sum(0)
    offsets = np.concatenate([[0], np.cumsum(kept)]).astype(np.int32)
    recv_dst = -np.ones(max(n_recv, 1), np.int32)
    # rows_cap as the CUDA wrapper sizes it (an upper bound under a capacity); the entries
    # past the kept rows are -1
    rows_cap = n_recv if capacity <= 0 else min(n_recv, capacity * El)
    row_src = -np.ones(max(rows_cap, int(offsets[-1]), 1), np.int32)
    r = 0
    for s in range(ws):
        for le in range(El):
            before = kept_seg[:s, le].sum()
            for i in range(rc[s, le]):
                if capacity <= 0 or base[s, le] + i < capacity:
                    dst = offsets[le] + before + i
                    recv_dst[r] = dst
                    row_src[dst] = r
                r += 1
    return dict(counts=torch.from_numpy(tot.astype(np.int32)), offsets=torch.from_numpy(offsets),
                row_src=torch.from_numpy(row_src), recv_dst=torch.from_numpy(recv_dst),
                rows_cap=int(max(rows_cap, 1)))


def combine(y, slot_row, w, T, k, shared=None, out=None):
    sr = slot_row.numpy().reshape(T, k)
    yn = y.numpy().astype(np.float64)
    wn = w.numpy()
    o = np.zeros((T, y.shape[1]))
    for j in range(k):
        m = sr[:, j] >= 0
        o[m] += wn[m, j, None] * yn[sr[m, j]]
    if shared is not None:
        o += shared.numpy()
    res = torch.from_numpy(o.astype(np.float32))
    if out is not None:
        out.copy_(res)
        return out
    return res


def ep_return_rows(row_src, offsets, recv_dst, n_recv, seg_table, row_bytes, rows_cap):
    seg = seg_table.numpy().astype(np.int64)
    nsrc = (seg.size - 1) // 2
    starts, base = seg[:nsrc + 1], seg[nsrc + 1:]

    def addr(r):
        s = int(np.searchsorted(starts[:nsrc], r, side="right")) - 1
        return int(base[s]) + (r - int(starts[s])) * row_bytes

    kept = int(offsets.numpy()[-1])
    rs = row_src.numpy() if row_src is not None else np.arange(max(rows_cap, 1))
    ptrs = np.zeros(max(rows_cap, 1), np.int64)
    for i in range(min(kept, rows_cap)):
        r = int(rs[i])
        if 0 <= r < n_recv:
            ptrs[i] = addr(r)
    if recv_dst is not None:
        rd = recv_dst.numpy()
        for r in range(n_recv):
            if rd[r] < 0:
                ctypes.memset(addr(r), 0, row_bytes)
    return torch.from_numpy(ptrs)


def ep_dedup_ranks(idx, El, ws, rank):
    it = idx.numpy()
    T, k = it.shape
    r = it // El
    ridx = -np.ones((T, k), np.int32)
    for t in range(T):
        for j in range(k):
            if r[t, j] not in r[t, :j]:
                ridx[t, j] = (r[t, j] - rank) % ws
    return torch.from_numpy(ridx)


def ep_dedup_meta(idx, w, ridx, slot_row, own_count, El, ws, rows_cap):
    it, wn, rn = idx.numpy(), w.numpy(), ridx.numpy()
    sr = slot_row.numpy().reshape(it.shape)
    T, k = it.shape
    meta_e = -np.ones((max(rows_cap, 1), k), np.int32)
    meta_w = np.zeros((max(rows_cap, 1), k), np.float32)
    own_e = -np.ones((max(T, 1), k), np.int32)
    for t in range(T):
        for j in range(k):
            if rn[t, j] < 0 or sr[t, j] < 0:
                continue
            p = sr[t, j]
            same = it[t] // El == it[t, j] // El
            meta_e[p] = np.where(same, it[t] % El, -1)
            meta_w[p] = np.where(same, wn[t], 0.0)
            if rn[t, j] == 0:
                own_e[p] = meta_e[p]
    return torch.from_numpy(meta_e), torch.from_numpy(meta_w), torch.from_numpy(own_e)


def ep_layout(counts_all, rank, capacity, recv_base, ret_base, row_bytes, recv_rows_max, out, rotated=False):
    Gin = counts_all.numpy().astype(np.int64)
    ws, E = Gin.shape
    El, me = E // ws, rank
    rot = rotated and El == 1
    # rotated: row s of the input counts source s's groups g = destination (s + g) % ws
    G = np.stack([np.roll(Gin[s_], s_) for s_ in range(ws)]) if rot else Gin
    before = np.cumsum(G, 0) - G
    Kp = np.clip(capacity - before, 0, G) if capacity > 0 else G.copy()
    owner = np.arange(E) // El
    per_exp = (Kp * (owner[None, :] != np.arange(ws)[:, None])).sum(0)
    eo = np.zeros(E, np.int64)
    n_recv = np.zeros(ws, np.int64)
    for r in range(ws):
        seg = per_exp[r * El:(r + 1) * El]
        eo[r * El:(r + 1) * El] = np.cumsum(seg) - seg
        n_recv[r] = seg.sum()
    overflow = bool((n_recv > recv_rows_max).any())
    rbase, tbase = recv_base.numpy(), ret_base.numpy()
    send_addr = np.zeros(E, np.int64)
    keep = np.zeros(E, np.int32)
    for e in range(E):
        so = sum(int(Kp[s, e]) for s in range(me) if s != owner[e])
        o = (e - me) % ws if rot else e
        if owner[e] != me and not overflow:
            send_addr[o] = int(rbase[owner[e]]) + int(eo[e] + so) * row_bytes
        keep[o] = 0 if overflow else Kp[me, e]
    nseg = El * ws
    seg = np.zeros(2 * nseg + 1, np.int64)
    for i in range(nseg):
        le, s = divmod(i, ws)
        e = me * El + le
        so = sum(int(Kp[q, e]) for q in range(s) if q != me)
        seg[i] = 0 if overflow else eo[e] + so
        pos = (e - s) % ws if rot else e
        seg[nseg + 1 + i] = int(tbase[s]) + int(Gin[s, :pos].sum() if rot else G[s, :e].sum()) * row_bytes
    seg[nseg] = 0 if overflow else n_recv[me]
    roff = np.concatenate([eo[me * El:(me + 1) * El], [n_recv[me]]]) if not overflow else np.zeros(El + 1)
    out["send_addr"].copy_(torch.from_numpy(send_addr))
    out["keep"].copy_(torch.from_numpy(keep))
    out["recv_offsets"].copy_(torch.from_numpy(roff.astype(np.int32)))
    out["seg"].copy_(torch.from_numpy(seg))
    return out


def ep_send_rows(x, row_token, offsets, own_first, own_count, send_addr, keep, rows_cap):
    off = offsets.numpy().astype(np.int64)
    E = off.size - 1
    rt, sa, kp = row_token.numpy(), send_addr.numpy(), keep.numpy()
    if x.shape[0] == 0:
        return
    xr = np.ascontiguousarray(x.contiguous().view(torch.uint8).numpy().reshape(x.shape[0], -1))   # rows as bytes
    rb = xr.shape[1]
    for i in range(int(off[E])):
        if off[own_first] <= i < off[own_first + own_count]:
            continue
        e = int(np.searchsorted(off[:E], i, side="right")) - 1
        p = i - int(off[e])
        if p >= kp[e] or sa[e] == 0 or rt[i] < 0:
            continue
        ctypes.memmove(int(sa[e]) + p * rb, xr[rt[i]].ctypes.data, rb)


def ep_drop_slots(idx, offsets, keep, slot_row):
    it, off, kp = idx.numpy().reshape(-1), offsets.numpy(), keep.numpy()
    sr = slot_row.numpy().reshape(-1)
    for s in range(it.size):
        e, r = int(it[s]), int(sr[s])
        if 0 <= e < kp.size and r >= 0 and r - off[e] >= kp[e]:
            sr[s] = -1


def ep_clear_tail(idx, n_rows):
    n = int(n_rows.numpy().reshape(-1)[0])
    idx.numpy()[n:] = -1


def store_rows(src, row_ptrs, n_rows):
    sb = np.ascontiguousarray(src.contiguous().view(torch.uint8).numpy().reshape(src.shape[0], -1))
    ptr = row_ptrs.numpy()
    for r in range(n_rows):
        if ptr[r]:
            ctypes.memmove(int(ptr[r]), sb[r].ctypes.data, sb.shape[1])


def copy_rows_count(dst, src, n_rows):
    n = int(n_rows.numpy().reshape(-1)[0])
    dst[:n] = src[:n]


# ---- the layer backward's kernels (expert-parallel backward on gloo ranks)

def router(x, gate_w, k, logit_bias=None, return_logits=False):
    xn = x.numpy().astype(np.float32)
    lg = xn @ gate_w.numpy().astype(np.float32).T
    lb = lg + (logit_bias.numpy() if logit_bias is not None else 0)
    T, E = lg.shape
    idx = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-lb[t, e], e))[:k]
        v = lb[t, order]
        ex = np.exp(v - v[0])
        idx[t], w[t] = order, ex / ex.sum()
    res = (torch.from_numpy(idx), torch.from_numpy(w))
    return res + (torch.from_numpy(lg),) if return_logits else res


def transpose_batched(src, out=None):
    return src.transpose(1, 2).contiguous()


def grouped_gemm(A, B, offsets, *, B3=None, epilogue=0, out_dtype=None, out=None, ends=None, row_ptrs=None):
    An, Bn = A.numpy().astype(np.float64), B.numpy().astype(np.float64)
    rows_cap, (G, N, _) = An.shape[0], Bn.shape
    off = offsets.numpy()
    width = 2 * N if epilogue == 3 else N
    C = np.zeros((max(rows_cap, 1), width))
    for g in range(G):
        r0, r1 = min(max(int(off[g]), 0), rows_cap), min(max(int(off[g + 1]), 0), rows_cap)
        if r1 <= r0:
            continue
        a = An[r0:r1] @ Bn[g].T
        if epilogue == 0:
            C[r0:r1] = a
        else:
            b = An[r0:r1] @ B3.numpy().astype(np.float64)[g].T
            C[r0:r1] = np.concatenate([a, b], 1) if epilogue == 3 else a / (1 + np.exp(-a)) * b
    res = torch.from_numpy(C.astype(np.float32))
    if out is not None:
        out[:res.shape[0]].copy_(res[:out.shape[0]])
        return out
    return res


def swiglu_bwd(ab, g, row_w, n_rows, dw_row):
    abn, gn = ab.numpy(), g.numpy()
    rows = int(n_rows[0]) if n_rows is not None else gn.shape[0]
    F = gn.shape[1]
    a, b, gg = abn[:rows, :F].astype(np.float64), abn[:rows, F:].astype(np.float64), gn[:rows].astype(np.float64)
    wr = row_w.numpy()[:rows, None].astype(np.float64) if row_w is not None else 1.0
    sg = 1 / (1 + np.exp(-a))
    si = a * sg
    h = si * b
    dh = wr * gg
    if dw_row is not None:
        dw_row.numpy()[:rows] = (gg * h).sum(1)
    abn[:rows, :F] = dh * b * sg * (1 + a * (1 - sg))
    abn[:rows, F:] = dh * si
    gn[:rows] = wr * h


def linear_bwd(g, xr, dr, row_w, n_rows, dw_row):
    rows = int(n_rows[0])
    gn, xn, dn = g.numpy(), xr.numpy(), dr.numpy()
    wr = row_w.numpy()[:rows, None]
    dw_row.numpy()[:rows] = (gn[:rows].astype(np.float64) * xn[:rows]).sum(1)
    gn[:rows] = wr * gn[:rows]
    dn[:rows] = wr * dn[:rows]


def wgrad_gemm_rows(A, B, k_offsets, M=None, N=None, out=None):
    An, Bn = A.numpy().astype(np.float64), B.numpy().astype(np.float64)
    M = An.shape[1] if M is None else M
    N = Bn.shape[1] if N is None else N
    off = k_offsets.numpy()
    G = off.shape[0] - 1
    C = np.zeros((G, M, N))
    for g in range(G):
        k0, k1 = int(off[g]), int(off[g + 1])
        C[g] = An[k0:k1, :M].T @ Bn[k0:k1, :N]
    return torch.from_numpy(C.astype(np.float32))


def moe_bwd_dx(dxr, slot_row, idx, w, dw_row, gate_w, dxs, dx, slot_row_full=None, dsel_row=None):
    T, k = idx.shape
    sr = slot_row.numpy().reshape(T, k)
    idn, wn = idx.numpy(), w.numpy().astype(np.float64)
    dxrn, dwn, gn = dxr.numpy().astype(np.float64), dw_row.numpy().astype(np.float64), gate_w.numpy()
    dwj = np.where(sr >= 0, dwn[np.maximum(sr, 0)], 0.0)
    ds = wn * (dwj - (wn * dwj).sum(1, keepdims=True))
    acc = np.zeros((T, dx.shape[1]))
    for j in range(k):
        m = sr[:, j] >= 0
        acc[m] += dxrn[sr[m, j]]
        acc += ds[:, j, None] * gn[idn[:, j]]
    if dxs is not None:
        acc += dxs.numpy()
    dx.copy_(torch.from_numpy(acc.astype(np.float32)))
    if dsel_row is not None:
        srf = slot_row_full.numpy().reshape(T, k)
        dsel_row.numpy()[srf[srf >= 0]] = ds[srf >= 0]


def router_dwg(x, row_token_full, offsets_full, dsel_row, E, out=None):
    xn, rt, off, ds = x.numpy().astype(np.float64), row_token_full.numpy(), offsets_full.numpy(), dsel_row.numpy()
    G = np.zeros((E, xn.shape[1]))
    for e in range(E):
        for r in range(int(off[e]), int(off[e + 1])):
            G[e] += ds[r] * xn[rt[r]]
    return torch.from_numpy(G.astype(np.float32))
