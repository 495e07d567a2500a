"""Tensor-level wrappers over the C ABI.  Each function checks its tensors (CUDA,
contiguous, dtype), allocates outputs with torch and calls exactly one libswiftmoe
entry point on the current CUDA stream.  They never fall back to another
implementation: a non-CUDA tensor or a failed call raises."""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib as L


def _need_cuda(*ts):
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise L.SwiftMoEError("swiftmoe_b200 kernels need CUDA tensors (no CPU fallback)")
            if not t.is_contiguous():
                raise L.SwiftMoEError("swiftmoe_b200 kernels need contiguous tensors")


def _workspace(device, nbytes: int) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def router(x: torch.Tensor, gate_w: torch.Tensor, k: int, logit_bias: Optional[torch.Tensor] = None,
           return_logits: bool = False):
    """idx [T,k] int32, w [T,k] fp32 (and fp32 gate logits [T,E] before the offsets)."""
    _need_cuda(x, gate_w, logit_bias)
    T, d = x.shape
    E = gate_w.shape[0]
    if gate_w.dtype != x.dtype:
        raise L.SwiftMoEError("gate weight dtype must match x")
    lib = L.load()
    dt = L.dtype_code(x.dtype)
    idx = torch.empty((T, k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, k), dtype=torch.float32, device=x.device)
    logits = torch.empty((T, E), dtype=torch.float32, device=x.device) if return_logits else None
    ws = _workspace(x.device, lib.smoe_router_workspace_size(T, d, E, dt))
    bias = logit_bias.float().contiguous() if logit_bias is not None else None
    L.check(lib.smoe_router_fwd(L.ptr(x), L.ptr(gate_w), dt, L.ptr(bias), T, d, E, k, L.ptr(idx), L.ptr(w),
                                L.ptr(logits), L.ptr(ws), ws.numel(), L.stream_handle(x.device)), "smoe_router_fwd")
    return (idx, w, logits) if return_logits else (idx, w)


def topk_from_logits(logits: torch.Tensor, k: int):
    _need_cuda(logits)
    if logits.dtype != torch.float32:
        raise L.SwiftMoEError("logits must be float32")
    T, E = logits.shape
    idx = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    L.check(L.load().smoe_topk_from_logits(L.ptr(logits), T, E, k, L.ptr(idx), L.ptr(w),
                                           L.stream_handle(logits.device)), "smoe_topk_from_logits")
    return idx, w


def dispatch_plan(idx: torch.Tensor, num_experts: int, capacity: int = 0, row_align: int = 1):
    """Returns dict(counts [E], offsets [E+1], slot_row [T*k], row_token [rows_cap], rows_cap)."""
    _need_cuda(idx)
    if idx.dtype != torch.int32:
        raise L.SwiftMoEError("idx must be int32")
    T, k = idx.shape
    E = num_experts
    lib = L.load()
    rows_cap = int(lib.smoe_plan_rows_cap(T, k, E, capacity, row_align))
    dev = idx.device
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    slot_row = torch.empty(T * k, dtype=torch.int32, device=dev)
    row_token = torch.empty(max(rows_cap, 1), dtype=torch.int32, device=dev)
    ws = _workspace(dev, lib.smoe_plan_workspace_size(T, k, E))
    L.check(lib.smoe_dispatch_plan(L.ptr(idx), T, k, E, capacity, row_align, L.ptr(counts), L.ptr(offsets),
                                   L.ptr(slot_row), L.ptr(row_token), max(rows_cap, 1), L.ptr(ws), ws.numel(),
                                   L.stream_handle(dev)), "smoe_dispatch_plan")
    return dict(counts=counts, offsets=offsets, slot_row=slot_row, row_token=row_token, rows_cap=rows_cap)


def permute_rows(x: torch.Tensor, row_token: torch.Tensor, offsets: torch.Tensor, rows_cap: int,
                 out: Optional[torch.Tensor] = None):
    _need_cuda(x, row_token, offsets)
    T, d = x.shape
    E = offsets.numel() - 1
    if out is None:
        out = torch.empty((max(rows_cap, 1), d), dtype=x.dtype, device=x.device)
    L.check(L.load().smoe_permute_rows(L.ptr(x), L.dtype_code(x.dtype), T, d, L.ptr(row_token), L.ptr(offsets), E,
                                       rows_cap, L.ptr(out), L.stream_handle(x.device)), "smoe_permute_rows")
    return out


def gather_rows(src: torch.Tensor, index: torch.Tensor, n_rows: int, out: Optional[torch.Tensor] = None):
    _need_cuda(src, index)
    d = src.shape[1]
    if out is None:
        out = torch.empty((max(n_rows, 1), d), dtype=src.dtype, device=src.device)
    L.check(L.load().smoe_gather_rows(L.ptr(src), L.dtype_code(src.dtype), d, L.ptr(index), n_rows, L.ptr(out),
                                      L.stream_handle(src.device)), "smoe_gather_rows")
    return out


def combine(y: torch.Tensor, slot_row: torch.Tensor, w: torch.Tensor, T: int, k: int,
            shared: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
    _need_cuda(y, slot_row, w, shared)
    d = y.shape[1]
    if out is None:
        out = torch.empty((T, d), dtype=y.dtype, device=y.device)
    L.check(L.load().smoe_combine(L.ptr(y), L.dtype_code(y.dtype), L.ptr(slot_row), L.ptr(w), T, k, d,
                                  L.ptr(shared), L.ptr(out), L.stream_handle(y.device)), "smoe_combine")
    return out


def grouped_gemm(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor, *, B3: Optional[torch.Tensor] = None,
                 epilogue: int = L.SMOE_EPI_STORE, out_dtype: Optional[torch.dtype] = None,
                 out: Optional[torch.Tensor] = None, ends: Optional[torch.Tensor] = None,
                 row_ptrs: Optional[torch.Tensor] = None):
    """C[rows_cap, N] for groups of rows [offsets[g], offsets[g+1]) -- or [offsets[g],
    ends[g]) when ``ends`` is given -- of A; B is [G, N, K].

    ``row_ptrs`` (int64 [rows_cap] device addresses, see ``ep_return_rows``): output row
    r is stored at row_ptrs[r] instead (possibly another GPU's memory); returns None."""
    _need_cuda(A, B, B3, offsets, ends, row_ptrs)
    rows_cap, K = A.shape
    G, N, K2 = B.shape
    if K2 != K:
        raise L.SwiftMoEError("K mismatch")
    od = out_dtype or A.dtype
    if row_ptrs is not None:
        if row_ptrs.dtype != torch.int64 or row_ptrs.numel() < rows_cap:
            raise L.SwiftMoEError("row_ptrs must be int64 with one address per row of A")
        L.check(L.load().smoe_grouped_gemm_rows(L.ptr(A), L.ptr(B), L.ptr(B3), L.ptr(row_ptrs), L.dtype_code(A.dtype),
                                                L.dtype_code(od), epilogue, L.ptr(offsets), L.ptr(ends), G, rows_cap,
                                                N, K, L.stream_handle(A.device)), "smoe_grouped_gemm_rows")
        return None
    if out is None:
        out = torch.empty((max(rows_cap, 1), N), dtype=od, device=A.device)
    L.check(L.load().smoe_grouped_gemm(L.ptr(A), L.ptr(B), L.ptr(B3), L.ptr(out), L.dtype_code(A.dtype),
                                       L.dtype_code(od), epilogue, L.ptr(offsets), L.ptr(ends), G, rows_cap, N, K,
                                       L.stream_handle(A.device)), "smoe_grouped_gemm")
    return out


def wgrad_gemm(A: torch.Tensor, B: torch.Tensor, k_offsets: torch.Tensor, K: Optional[int] = None,
               out: Optional[torch.Tensor] = None):
    """C[g] = A[:, K_g] @ B[:, K_g]^T (fp32 [G, M, N]) for the K ranges K_g = [k_offsets[g],
    k_offsets[g+1]) of the K-major 16-bit operands A [M, ld] and B [N, ld] (the first K
    columns; group starts multiples of 64)."""
    _need_cuda(A, B, k_offsets)
    M, lda = A.shape
    N, ldb = B.shape
    G = k_offsets.numel() - 1
    K = min(lda, ldb) if K is None else K
    if out is None:
        out = torch.empty((G, M, N), dtype=torch.float32, device=A.device)
    L.check(L.load().smoe_wgrad_gemm(L.ptr(A), lda, L.ptr(B), ldb, L.dtype_code(A.dtype), L.ptr(k_offsets), G, M, N,
                                     K, L.ptr(out), L.stream_handle(A.device)), "smoe_wgrad_gemm")
    return out


def wgrad_gemm_rows(A: torch.Tensor, B: torch.Tensor, k_offsets: torch.Tensor, M: Optional[int] = None,
                    N: Optional[int] = None, out: Optional[torch.Tensor] = None):
    """C[g] = A[K_g, :M]^T @ B[K_g, :N] (fp32 [G, M, N]) for the row ranges K_g =
    [k_offsets[g], k_offsets[g+1]) of the row-major 16-bit operands A [K, lda], B [K, ldb]."""
    _need_cuda(A, B, k_offsets)
    K, lda = A.shape
    K2, ldb = B.shape
    M = lda if M is None else M
    N = ldb if N is None else N
    G = k_offsets.numel() - 1
    if out is None:
        out = torch.empty((G, M, N), dtype=torch.float32, device=A.device)
    L.check(L.load().smoe_wgrad_gemm_rows(L.ptr(A), lda, L.ptr(B), ldb, L.dtype_code(A.dtype), L.ptr(k_offsets), G,
                                          M, N, min(K, K2), L.ptr(out), L.stream_handle(A.device)),
            "smoe_wgrad_gemm_rows")
    return out


def swiglu_bwd(ab: torch.Tensor, g: torch.Tensor, row_w: Optional[torch.Tensor], n_rows: Optional[torch.Tensor],
               dw_row: Optional[torch.Tensor]) -> None:
    """SwiGLU backward of the routed rows, in place: ab [rows, 2F] = [a | b] -> [da | db],
    g [rows, F] (dout_r W2) -> w_r * h, dw_row[r] = <g_r, h_r>; rows r < n_rows[0] (device
    int32, None: all); row_w fp32 [rows] (None: 1)."""
    _need_cuda(ab, g, row_w, n_rows, dw_row)
    rows_cap, F = g.shape
    L.check(L.load().smoe_swiglu_bwd(L.ptr(ab), L.ptr(g), L.ptr(row_w), L.ptr(n_rows), rows_cap, F,
                                     L.dtype_code(g.dtype), L.ptr(dw_row), L.stream_handle(g.device)),
            "smoe_swiglu_bwd")


def linear_bwd(g: torch.Tensor, xr: torch.Tensor, dr: torch.Tensor, row_w: torch.Tensor, n_rows: torch.Tensor,
               dw_row: torch.Tensor) -> None:
    """Linear-expert backward of the routed rows, in place: dw_row[r] = <g_r, x_r>,
    g -> w_r g, dr -> w_r dr, for rows r < n_rows[0]."""
    _need_cuda(g, xr, dr, row_w, n_rows, dw_row)
    rows_cap, d = g.shape
    L.check(L.load().smoe_linear_bwd(L.ptr(g), L.ptr(xr), L.ptr(dr), L.ptr(row_w), L.ptr(n_rows), rows_cap, d,
                                     L.dtype_code(g.dtype), L.ptr(dw_row), L.stream_handle(g.device)),
            "smoe_linear_bwd")


def moe_bwd_dx(dxr: torch.Tensor, slot_row: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, dw_row: torch.Tensor,
               gate_w: torch.Tensor, dxs: Optional[torch.Tensor], dx: torch.Tensor,
               slot_row_full: Optional[torch.Tensor] = None, dsel_row: Optional[torch.Tensor] = None) -> None:
    """dx [T, d] from the slots' input-gradient rows dxr (at slot_row), the gate weights'
    gradients dw_row (per dxr row), the router backward and the shared expert's dxs."""
    _need_cuda(dxr, slot_row, idx, w, dw_row, gate_w, dxs, dx, slot_row_full, dsel_row)
    T, k = idx.shape
    d = dx.shape[1]
    L.check(L.load().smoe_moe_bwd_dx(L.ptr(dxr), L.ptr(slot_row), L.ptr(idx), L.ptr(w), L.ptr(dw_row), L.ptr(gate_w),
                                     L.ptr(dxs), T, k, d, L.dtype_code(dx.dtype), L.ptr(dx), L.ptr(slot_row_full),
                                     L.ptr(dsel_row), L.stream_handle(dx.device)), "smoe_moe_bwd_dx")


def router_dwg(x: torch.Tensor, row_token_full: torch.Tensor, offsets_full: torch.Tensor, dsel_row: torch.Tensor,
               E: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gate gradient fp32 [E, d] from dsel per row of a plan over every slot."""
    _need_cuda(x, row_token_full, offsets_full, dsel_row)
    d = x.shape[1]
    lib = L.load()
    ws = torch.empty(max(int(lib.smoe_router_dwg_workspace_size(d, E)), 1), dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty((E, d), dtype=torch.float32, device=x.device)
    L.check(lib.smoe_router_dwg(L.ptr(x), L.ptr(row_token_full), L.ptr(offsets_full), L.ptr(dsel_row), d, E,
                                L.dtype_code(x.dtype), L.ptr(out), L.ptr(ws), ws.numel(), L.stream_handle(x.device)),
            "smoe_router_dwg")
    return out


def tf32_split_weights(w: torch.Tensor) -> torch.Tensor:
    """fp32 [..., K] -> [..., 3K] rows [lo | hi | hi] (hi: the tf32 rounding, lo: the exact
    remainder), the weight layout of the fp32 GEMMs on the tf32 tensor cores
    (``smoe_tf32_split_weights``); K % 4 == 0."""
    _need_cuda(w)
    if w.dtype != torch.float32:
        raise L.SwiftMoEError("tf32_split_weights takes fp32 weights")
    w = w.contiguous()
    Kd = w.shape[-1]
    out = torch.empty(tuple(w.shape[:-1]) + (3 * Kd,), dtype=torch.float32, device=w.device)
    L.check(L.load().smoe_tf32_split_weights(L.ptr(w), L.ptr(out), w.numel() // max(Kd, 1), Kd,
                                             L.stream_handle(w.device)), "smoe_tf32_split_weights")
    return out


def transpose_batched(src: torch.Tensor, out: Optional[torch.Tensor] = None):
    """[G, R, C] -> [G, C, R]."""
    _need_cuda(src)
    G, R, Cc = src.shape
    if out is None:
        out = torch.empty((G, Cc, R), dtype=src.dtype, device=src.device)
    L.check(L.load().smoe_transpose_batched(L.ptr(src), L.ptr(out), L.dtype_code(src.dtype), G, R, Cc,
                                            L.stream_handle(src.device)), "smoe_transpose_batched")
    return out


def ep_regroup_plan(recv_counts: torch.Tensor, capacity: int, n_recv: int, pos_base: Optional[torch.Tensor] = None):
    """recv_counts [ws, E_l] int32 -> dict(counts, offsets, row_src, recv_dst, rows_cap).

    pos_base [ws, E_l] int32 (optional): global position of each segment's first row in
    its expert's (source rank, token, slot) order, when the batch travels in chunks."""
    _need_cuda(recv_counts, pos_base)
    ws_, El = recv_counts.shape
    lib = L.load()
    dev = recv_counts.device
    rows_cap = n_recv if capacity <= 0 else min(n_recv, capacity * El)
    counts = torch.empty(El, dtype=torch.int32, device=dev)
    offsets = torch.empty(El + 1, dtype=torch.int32, device=dev)
    # the plan writes row_src for the kept rows only; the rest of rows_cap (an upper bound
    # under a capacity) holds -1, "no row", for readers that take all rows_cap entries
    row_src = torch.full((max(rows_cap, 1),), -1, dtype=torch.int32, device=dev)
    recv_dst = torch.empty(max(n_recv, 1), dtype=torch.int32, device=dev)
    wsb = _workspace(dev, lib.smoe_ep_regroup_workspace_size(ws_, El))
    L.check(lib.smoe_ep_regroup_plan(L.ptr(recv_counts), ws_, El, capacity, L.ptr(pos_base), n_recv, L.ptr(counts),
                                     L.ptr(offsets),
                                     L.ptr(row_src), L.ptr(recv_dst), L.ptr(wsb), wsb.numel(), L.stream_handle(dev)),
            "smoe_ep_regroup_plan")
    return dict(counts=counts, offsets=offsets, row_src=row_src, recv_dst=recv_dst, rows_cap=rows_cap)


def ep_return_rows(row_src: torch.Tensor, offsets: torch.Tensor, recv_dst: torch.Tensor, n_recv: int,
                   seg_table: torch.Tensor, row_bytes: int, rows_cap: int) -> torch.Tensor:
    """Return address of every expert row (int64 [rows_cap]) for ``grouped_gemm(row_ptrs=)``;
    zero rows at the return addresses of dropped received rows.  row_src None: expert
    row i is received row i; recv_dst None: nothing dropped.  seg_table: int64
    [2 * n_src + 1] device tensor: source segment starts (n_src + 1, last = n_recv), then
    the address of each source's return region."""
    _need_cuda(row_src, offsets, recv_dst, seg_table)
    El = offsets.numel() - 1
    dev = offsets.device
    n_src = (seg_table.numel() - 1) // 2
    row_ptrs = torch.empty(max(rows_cap, 1), dtype=torch.int64, device=dev)
    L.check(L.load().smoe_ep_return_rows(L.ptr(row_src), L.ptr(offsets), El, L.ptr(recv_dst), n_recv,
                                         L.ptr(seg_table), n_src, row_bytes, L.ptr(row_ptrs), rows_cap,
                                         L.stream_handle(dev)), "smoe_ep_return_rows")
    return row_ptrs


def ep_layout(counts_all: torch.Tensor, rank: int, capacity: int, recv_base: torch.Tensor, ret_base: torch.Tensor,
              row_bytes: int, recv_rows_max: int, out: dict, rotated: bool = False):
    """Device-side layout of the exchange from the all-gathered counts [ws, E] (see
    smoe_ep_layout).  ``out`` holds the preallocated outputs: send_addr [E] int64, keep [E]
    int32, recv_offsets [E_l+1] int32, seg [2*E_l*ws+1] int64; returns it."""
    _need_cuda(counts_all, recv_base, ret_base)
    ws_, E = counts_all.shape
    L.check(L.load().smoe_ep_layout(L.ptr(counts_all), ws_, E, rank, capacity, L.ptr(recv_base), L.ptr(ret_base),
                                    row_bytes, recv_rows_max, L.ptr(out["send_addr"]), L.ptr(out["keep"]),
                                    L.ptr(out["recv_offsets"]), L.ptr(out["seg"]), 1 if rotated else 0,
                                    L.stream_handle(counts_all.device)), "smoe_ep_layout")
    return out


def ep_clear_tail(idx: torch.Tensor, n_rows: torch.Tensor) -> None:
    """idx [rows_cap, k] slots of the rows r >= n_rows[0] (device) set to -1, in place."""
    _need_cuda(idx, n_rows)
    rows_cap, k = idx.shape
    L.check(L.load().smoe_ep_clear_tail(L.ptr(idx), L.ptr(n_rows), rows_cap, k, L.stream_handle(idx.device)),
            "smoe_ep_clear_tail")


def store_rows(src: torch.Tensor, row_ptrs: torch.Tensor, n_rows: int) -> None:
    """Row r of src (r < n_rows) to the address row_ptrs[r] (0 = skip)."""
    _need_cuda(src, row_ptrs)
    L.check(L.load().smoe_store_rows(L.ptr(src), src.shape[1] * src.element_size(), L.ptr(row_ptrs), n_rows,
                                     L.stream_handle(src.device)), "smoe_store_rows")


def copy_rows_count(dst: torch.Tensor, src: torch.Tensor, n_rows: torch.Tensor) -> None:
    """dst rows [0, n_rows[0]) = src rows (n_rows in device memory)."""
    _need_cuda(dst, src, n_rows)
    rows_cap = min(dst.shape[0], src.shape[0])
    L.check(L.load().smoe_copy_rows_count(L.ptr(dst), L.ptr(src), src.shape[1] * src.element_size(), L.ptr(n_rows),
                                          rows_cap, L.stream_handle(src.device)), "smoe_copy_rows_count")


def ep_send_rows(x: torch.Tensor, row_token: torch.Tensor, offsets: torch.Tensor, own_first: int, own_count: int,
                 send_addr: torch.Tensor, keep: torch.Tensor, rows_cap: int) -> None:
    """Rows of the other ranks' experts from x straight into their receive buffers."""
    _need_cuda(x, row_token, offsets, send_addr, keep)
    E = offsets.numel() - 1
    L.check(L.load().smoe_ep_send_rows(L.ptr(x), x.shape[1] * x.element_size(), L.ptr(row_token), L.ptr(offsets), E,
                                       own_first, own_count, L.ptr(send_addr), L.ptr(keep), rows_cap,
                                       L.stream_handle(x.device)), "smoe_ep_send_rows")


def ep_drop_slots(idx: torch.Tensor, offsets: torch.Tensor, keep: torch.Tensor, slot_row: torch.Tensor) -> None:
    """slot_row[s] = -1 (in place) for the slots the capacity cut dropped."""
    _need_cuda(idx, offsets, keep, slot_row)
    E = offsets.numel() - 1
    L.check(L.load().smoe_ep_drop_slots(L.ptr(idx), idx.numel(), L.ptr(offsets), E, L.ptr(keep), L.ptr(slot_row),
                                        L.stream_handle(idx.device)), "smoe_ep_drop_slots")


def ep_dedup_ranks(idx: torch.Tensor, El: int, ws: int, rank: int) -> torch.Tensor:
    """ridx [T, k] int32: rotated destination rank of the first slot of each token bound
    for a rank, -1 for its later slots to the same rank (see smoe_ep_dedup_ranks)."""
    _need_cuda(idx)
    T, k = idx.shape
    ridx = torch.empty((T, k), dtype=torch.int32, device=idx.device)
    L.check(L.load().smoe_ep_dedup_ranks(L.ptr(idx), T, k, El, ws, rank, L.ptr(ridx),
                                         L.stream_handle(idx.device)), "smoe_ep_dedup_ranks")
    return ridx


def ep_dedup_meta(idx: torch.Tensor, w: torch.Tensor, ridx: torch.Tensor, slot_row: torch.Tensor,
                  own_count: torch.Tensor, El: int, ws: int, rows_cap: int):
    """(meta_e [rows_cap, k] int32, meta_w [rows_cap, k] fp32, own_e [T, k] int32) of the
    sent rows (see smoe_ep_dedup_meta); own_count: device int32, this rank's row count."""
    _need_cuda(idx, w, ridx, slot_row, own_count)
    T, k = idx.shape
    dev = idx.device
    meta_e = torch.empty((max(rows_cap, 1), k), dtype=torch.int32, device=dev)
    meta_w = torch.empty((max(rows_cap, 1), k), dtype=torch.float32, device=dev)
    own_e = torch.empty((max(T, 1), k), dtype=torch.int32, device=dev)
    L.check(L.load().smoe_ep_dedup_meta(L.ptr(idx), L.ptr(w), L.ptr(ridx), L.ptr(slot_row), L.ptr(own_count), T, k,
                                        El, ws, L.ptr(meta_e), L.ptr(meta_w), L.ptr(own_e), L.stream_handle(dev)),
            "smoe_ep_dedup_meta")
    return meta_e, meta_w, own_e


def read_device_error(device) -> int:
    import ctypes as C
    flag = C.c_int(0)
    L.check(L.load().smoe_read_device_error(C.byref(flag), L.stream_handle(device)), "smoe_read_device_error")
    return flag.value
