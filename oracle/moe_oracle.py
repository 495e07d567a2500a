"""CPU restatement (numpy) of SwiftMoE's MoE-layer forward -- TEST INFRASTRUCTURE ONLY.

This module is the oracle.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and there
only as the checker or as the timed CPU baseline.  The product path
(``swiftmoe_b200``) never imports it; it fails loudly when its CUDA library is absent.

Parity pin: the linear-expert, top-2 path is pinned against fixtures produced by the
reference's own ``StandardMoE`` / ``UltimateMoE(use_triton=False)`` (see
``tests/golden/make_golden.py``).  SwiGLU experts at k=2 are pinned by running the
reference's ``StandardMoE`` control flow with SwiGLU modules substituted into its
``experts`` list.  top-k != 2, capacity dropping, the shared expert and per-expert logit
offsets do not exist in the reference; for those the restatement below is the
definition ("parity unpinned by the reference").

Reference files cited (paths inside the SwiftMoE project):
  models/baseline_moe.py   StandardMoE   (_route_tokens :56-67, _dispatch_tokens :69-141,
                                          _expert_forward :143-164, _combine_tokens :166-189)
  models/ultimate_moe.py   UltimateMoE   (torch routing fallback :288-295,
                                          MoEAsyncCommHandler.dispatch :114-143,
                                          _expert_compute :222-252, combine :145-155)
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

__all__ = [
    "gate_logits", "topk_lower_index", "softmax_rows", "route", "expert_rank_local",
    "capacity_for", "dispatch_plan", "linear_expert_pre", "linear_expert_post",
    "swiglu_expert", "MoEParams", "moe_forward", "bf16_round", "f16_round",
]


# --------------------------------------------------------------------------- numerics
def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), out).astype(np.float32)


def f16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to float16 and back."""
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def silu(a: np.ndarray) -> np.ndarray:
    return a / (1.0 + np.exp(-a))


# --------------------------------------------------------------------------- routing
def gate_logits(x: np.ndarray, wg: np.ndarray, logit_bias: Optional[np.ndarray] = None,
                acc=np.float32) -> np.ndarray:
    """logits = x @ Wg^T  (+ per-expert offset).

    Follows ``models/baseline_moe.py:59`` (``self.gate(x)``, an ``nn.Linear`` without bias)
    and ``models/ultimate_moe.py:289`` (``torch.matmul(x, self.gate_weight.t())``).
    ``logit_bias`` is the per-expert offset extension (absent in the reference).
    """
    lg = np.asarray(x, dtype=acc) @ np.asarray(wg, dtype=acc).T
    if logit_bias is not None:
        lg = lg + np.asarray(logit_bias, dtype=acc)[None, :]
    return lg.astype(np.float32)


def topk_lower_index(logits: np.ndarray, k: int):
    """Top-k per row, values descending, ties broken toward the LOWER expert index.

    Restates ``torch.topk(gate_logits, k=2, dim=-1)`` (``models/baseline_moe.py:62``,
    ``models/ultimate_moe.py:290``): the same selected values as torch, NaN ranked above
    every number.  Among EQUAL values torch's CPU kernel orders by its partial-sort /
    nth_element pass, which is not index order; this restatement (and the GPU router)
    takes the lower expert index first, a deterministic rule.  Without ties the indices
    are identical to torch's.  Returns (values float32 [T,k], indices int32 [T,k]).
    """
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    if k > E:
        raise ValueError("k must be <= number of experts")
    if T == 0:
        return np.zeros((0, k), np.float32), np.zeros((0, k), np.int32)
    isnan = np.isnan(logits)
    vals = np.where(isnan, np.float32(0), logits)
    col = np.broadcast_to(np.arange(E), logits.shape)
    # lexsort: last key is primary.  NaN first, then larger value, then lower index.
    order = np.lexsort((col, -vals, ~isnan), axis=1)[:, :k]
    idx = order.astype(np.int32)
    v = np.take_along_axis(logits, order, axis=1)
    return v.astype(np.float32), idx


def softmax_rows(v: np.ndarray) -> np.ndarray:
    """``torch.softmax(top_k_logits, dim=-1)`` (``models/baseline_moe.py:65``) in float32."""
    v = np.asarray(v, dtype=np.float32)
    if v.shape[0] == 0:
        return v.copy()
    m = np.max(v, axis=1, keepdims=True)
    e = np.exp(v - m, dtype=np.float32)
    return (e / np.sum(e, axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)


def route(x, wg, k=2, logit_bias=None):
    """Router: logits -> top-k -> softmax over the k selected logits.

    ``models/baseline_moe.py:56-67`` / ``models/ultimate_moe.py:288-293``.
    Returns (idx int32 [T,k], weights float32 [T,k], logits float32 [T,E]).
    """
    lg = gate_logits(x, wg, logit_bias)
    v, idx = topk_lower_index(lg, k)
    return idx, softmax_rows(v), lg


def expert_rank_local(idx: np.ndarray, num_experts: int, ws: int):
    """``target_rank = e // E_l``, ``local = e % E_l`` (``models/ultimate_moe.py:93-96,294-295``)."""
    el = num_experts // ws
    return (idx // el).astype(np.int32), (idx % el).astype(np.int32)


# --------------------------------------------------------------------------- dispatch
def capacity_for(capacity_factor: Optional[float], tokens_global: int, k: int,
                 num_experts: int) -> Optional[int]:
    """Per-expert capacity ``C = ceil(cf * T_glob * k / E)`` (extension; None = unlimited)."""
    if capacity_factor is None:
        return None
    return int(math.ceil(capacity_factor * tokens_global * k / num_experts))


def dispatch_plan(idx_per_rank: Sequence[np.ndarray], num_experts: int, ws: int,
                  capacity: Optional[int] = None):
    """Which (src_rank, token, slot) rows each expert receives, in index order.

    The reference sorts slots by target rank (``models/ultimate_moe.py:120``) and then by
    local expert (``:224``); both argsorts are unstable, but the layer output does not
    depend on the order within an expert because every row is processed independently
    and ``argsort(sort_idx)`` (``:121,252``) restores it.  The restatement fixes the
    order to (src_rank, token, slot) ascending.  With a capacity, rows beyond ``capacity``
    in that order are dropped (extension).

    Returns a list over global experts of int arrays [n_e, 3] = (src_rank, token, slot)
    for kept rows, and per-rank boolean ``kept[T,k]`` masks.
    """
    rows: List[list] = [[] for _ in range(num_experts)]
    kept = []
    for r, idx in enumerate(idx_per_rank):
        idx = np.asarray(idx)
        keep = np.zeros(idx.shape, dtype=bool)
        T, k = idx.shape
        for t in range(T):
            for j in range(k):
                e = int(idx[t, j])
                if capacity is None or len(rows[e]) < capacity:
                    rows[e].append((r, t, j))
                    keep[t, j] = True
        kept.append(keep)
    out = [np.asarray(v, dtype=np.int64).reshape(-1, 3) for v in rows]
    return out, kept


# --------------------------------------------------------------------------- experts
def linear_expert_pre(x, w, W, acc=np.float32):
    """UltimateMoE expert: ``torch.mm(x * w, W_e)`` (``models/ultimate_moe.py:245-249``).

    ``W`` is ``expert_weights[e]`` in the reference's ``x @ W`` layout [d_in, d_out]."""
    return (np.asarray(x, acc) * np.asarray(w, acc)[:, None]) @ np.asarray(W, acc)


def linear_expert_post(x, w, Wlin, acc=np.float32):
    """StandardMoE expert: ``self.experts[i](x) * w`` (``models/baseline_moe.py:159-162``).

    ``Wlin`` is ``nn.Linear.weight`` [d_out, d_in]."""
    return (np.asarray(x, acc) @ np.asarray(Wlin, acc).T) * np.asarray(w, acc)[:, None]


def swiglu_expert(x, w1, w3, w2, acc=np.float32, round_hidden=None):
    """SwiGLU expert ``w2(silu(w1 x) * w3 x)`` (extension; nn.Linear layouts).

    w1, w3: [F, d]; w2: [d, F].  ``round_hidden`` optionally rounds the hidden activation
    and the expert output to the storage dtype of a 16-bit pipeline (a bf16/fp16 layer
    keeps both in the compute dtype between its GEMMs, as the reference's torch path does
    for every intermediate)."""
    x = np.asarray(x, acc)
    h = silu(x @ np.asarray(w1, acc).T) * (x @ np.asarray(w3, acc).T)
    if round_hidden is not None:
        h = round_hidden(h.astype(np.float32)).astype(acc)
    y = h @ np.asarray(w2, acc).T
    if round_hidden is not None:
        y = round_hidden(y.astype(np.float32)).astype(acc)
    return y


# --------------------------------------------------------------------------- layer
@dataclass
class MoEParams:
    """Global (all-rank) parameters of one MoE layer, float32 numpy arrays.

    gate: [E, d].  Linear experts: ``expert_w[E, d, d]`` in the ``x @ W`` layout
    (UltimateMoE ``expert_weights``; StandardMoE's ``experts[i].weight`` is its
    transpose).  SwiGLU experts: ``w1, w3 [E, F, d]``, ``w2 [E, d, F]``.  Shared expert
    (SwiGLU): ``sw1, sw3 [S, Fs, d]``, ``sw2 [S, d, Fs]``.  ``logit_bias [E]`` optional.
    """
    gate: np.ndarray
    expert_type: str = "linear"
    expert_w: Optional[np.ndarray] = None
    w1: Optional[np.ndarray] = None
    w3: Optional[np.ndarray] = None
    w2: Optional[np.ndarray] = None
    sw1: Optional[np.ndarray] = None
    sw3: Optional[np.ndarray] = None
    sw2: Optional[np.ndarray] = None
    logit_bias: Optional[np.ndarray] = None
    extra: dict = field(default_factory=dict)

    @property
    def num_experts(self):
        return self.gate.shape[0]


def moe_forward(xs: Sequence[np.ndarray], p: MoEParams, *, ws: int = 1, k: int = 2,
                weighting: str = "post", capacity_factor: Optional[float] = None,
                acc=np.float32, round_hidden=None, return_aux: bool = False,
                capacity: Optional[int] = None, routing=None):
    """Full layer forward for ``ws`` ranks; ``xs[r]`` is rank r's [T_r, d] input.

    Control flow follows ``StandardMoE.forward`` (``models/baseline_moe.py:191-213``):
    route -> dispatch (rows grouped by owning rank / local expert) -> experts -> combine
    (``restored.view(M, k, d).sum(dim=1)``, slot order 0..k-1, ``:188-189``).
    ``weighting="pre"`` applies the gate weight before a linear expert as UltimateMoE
    does (``models/ultimate_moe.py:245``); ``"post"`` after it (``baseline_moe.py:162``).
    SwiGLU experts always use post-weighting.  Dropped rows contribute zero and the kept
    weights are not renormalised.  The shared expert output is added unweighted.
    ``round_hidden`` (e.g. ``bf16_round``) rounds the intermediates a 16-bit pipeline
    stores: the SwiGLU hidden activation and each expert's output before weighting.
    ``capacity`` (rows per expert, > 0) overrides the one derived from
    ``capacity_factor``, e.g. for ranks with unequal batches.
    ``routing`` (optional): per rank, the (idx [T,k], w [T,k]) to use instead of this
    restatement's own router -- e.g. the routing a device computed, so that dispatch,
    capacity cut, experts and combine are checked on exactly its decisions.
    """
    E = p.num_experts
    if E % ws:
        raise ValueError("num_experts must be divisible by world size")
    routed = []
    for r, x in enumerate(xs):
        if routing is not None:
            idx, w = routing[r]
            routed.append((np.asarray(idx, np.int64), np.asarray(w, np.float32), None))
            continue
        idx, w, lg = route(x, p.gate, k, p.logit_bias)
        routed.append((idx, w, lg))
    t_glob = sum(x.shape[0] for x in xs)
    cap = capacity_for(capacity_factor, t_glob, k, E)
    if capacity_factor is not None:
        # capacity is defined on the per-rank token count times ws (equal batches)
        cap = capacity_for(capacity_factor, xs[0].shape[0] * ws, k, E)
    if capacity is not None and capacity > 0:
        cap = capacity
    plan, kept = dispatch_plan([r[0] for r in routed], E, ws, cap)

    d = xs[0].shape[1] if len(xs) else p.gate.shape[1]
    outs = [np.zeros((x.shape[0], k, d), dtype=acc) for x in xs]
    for e in range(E):
        rows = plan[e]
        if rows.shape[0] == 0:
            continue
        xin = np.stack([xs[r][t] for (r, t, j) in rows]).astype(acc)
        wts = np.array([routed[r][1][t, j] for (r, t, j) in rows], dtype=acc)
        if p.expert_type == "linear":
            if weighting == "pre":
                y = linear_expert_pre(xin, wts, p.expert_w[e], acc)
            else:
                y = linear_expert_post(xin, np.ones_like(wts), p.expert_w[e].T, acc)
                if round_hidden is not None:
                    y = round_hidden(y.astype(np.float32)).astype(acc)
                y = y * wts[:, None]
        elif p.expert_type == "swiglu":
            y = swiglu_expert(xin, p.w1[e], p.w3[e], p.w2[e], acc, round_hidden) * wts[:, None]
        else:
            raise ValueError(p.expert_type)
        for n, (r, t, j) in enumerate(rows):
            outs[r][t, j] = y[n]
    results = []
    for r, x in enumerate(xs):
        o = np.zeros((x.shape[0], d), dtype=acc)
        for j in range(k):                       # slot order, as .sum(dim=1)
            o = o + outs[r][:, j, :]
        if p.sw1 is not None:
            for s in range(p.sw1.shape[0]):
                o = o + swiglu_expert(x, p.sw1[s], p.sw3[s], p.sw2[s], acc, round_hidden)
        results.append(o.astype(np.float32))
    if return_aux:
        return results, dict(routed=routed, plan=plan, kept=kept, capacity=cap)
    return results


# --------------------------------------------------------------------------- backward
def _swiglu_backward(xin, w1, w3, w2, dy, acc):
    """Gradients of ``y = w2(silu(w1 x) * w3 x)`` given dy: (dx, dw1, dw3, dw2)."""
    w1, w3, w2 = (np.asarray(a, acc) for a in (w1, w3, w2))
    g = xin @ w1.T
    u = xin @ w3.T
    s = 1.0 / (1.0 + np.exp(-g))
    h = g * s * u
    dh = dy @ w2
    dg = dh * u * s * (1.0 + g * (1.0 - s))      # d silu(g) / dg = s (1 + g (1 - s))
    du = dh * g * s
    return dg @ w1 + du @ w3, dg.T @ xin, du.T @ xin, dy.T @ h


def moe_backward(x: np.ndarray, p: MoEParams, dout: np.ndarray, *, k: int = 2, weighting: str = "post",
                 capacity_factor: Optional[float] = None, capacity: Optional[int] = None, acc=np.float64,
                 routing=None):
    """Gradients of one rank's layer output (``moe_forward`` with ws = 1) for the upstream
    gradient ``dout`` [T, d]: a dict with ``x``, ``gate`` and the expert weights in
    ``MoEParams`` layout (``expert_w``, or ``w1, w3, w2``; ``sw1, sw3, sw2`` for the shared
    expert).  Expert parallelism only moves rows, so the gradients of a multi-rank
    forward are these, rank by rank, with the capacity of the whole batch.

    The reference is forward-only; its torch ops differentiate as: top-k passes the
    gradient to the selected logits, ``softmax`` over them (``models/baseline_moe.py:62-65``),
    the expert ``Linear(x) * w`` (post-weighting, :159-162) or ``(x * w) @ W``
    (pre-weighting, ``models/ultimate_moe.py:245-249``), the k slots summed in slot order
    (:188-189).  Dropped slots (capacity) contribute 0 and stay in the softmax, as in the
    forward.  ``acc`` is the arithmetic precision (float64 by default).  ``routing``
    (optional): the (idx, w) to use instead of this restatement's router, as in
    ``moe_forward``."""
    x = np.asarray(x, acc)
    dout = np.asarray(dout, acc)
    T, d = x.shape
    E = p.num_experts
    if routing is not None:
        idx, w = np.asarray(routing[0], np.int64), np.asarray(routing[1], np.float32)
    else:
        idx, w, _ = route(x.astype(np.float32), p.gate, k, p.logit_bias)
    cap = capacity if capacity else capacity_for(capacity_factor, T, k, E)
    plan, _ = dispatch_plan([idx], E, 1, cap)
    wk = w.astype(acc)
    dw = np.zeros((T, k), acc)
    dx = np.zeros((T, d), acc)
    g = {}
    if p.expert_type == "linear":
        g["expert_w"] = np.zeros(p.expert_w.shape, acc)
    else:
        for n in ("w1", "w3", "w2"):
            g[n] = np.zeros(getattr(p, n).shape, acc)
    for e in range(E):
        rows = plan[e]
        if rows.shape[0] == 0:
            continue
        ts, js = rows[:, 1], rows[:, 2]
        xin, go, wts = x[ts], dout[ts], wk[ts, js][:, None]
        if p.expert_type == "linear":
            We = np.asarray(p.expert_w[e], acc)           # x @ W layout [d_in, d_out]
            if weighting == "pre":
                g["expert_w"][e] += (xin * wts).T @ go
                dxw = go @ We.T
                dw[ts, js] = (dxw * xin).sum(1)
                np.add.at(dx, ts, dxw * wts)
            else:
                y = xin @ We
                dw[ts, js] = (go * y).sum(1)
                g["expert_w"][e] += xin.T @ (go * wts)
                np.add.at(dx, ts, (go * wts) @ We.T)
        else:
            y = swiglu_expert(xin, p.w1[e], p.w3[e], p.w2[e], acc)
            dw[ts, js] = (go * y).sum(1)
            dxe, d1, d3, d2 = _swiglu_backward(xin, p.w1[e], p.w3[e], p.w2[e], go * wts, acc)
            g["w1"][e] += d1
            g["w3"][e] += d3
            g["w2"][e] += d2
            np.add.at(dx, ts, dxe)
    # softmax over the k selected logits, then top-k scatters back to the logits
    dv = wk * (dw - (wk * dw).sum(1, keepdims=True))
    dlog = np.zeros((T, E), acc)
    np.add.at(dlog, (np.repeat(np.arange(T), k), idx.reshape(-1)), dv.reshape(-1))
    gate = np.asarray(p.gate, acc)
    dx += dlog @ gate
    g["gate"] = dlog.T @ x
    if p.sw1 is not None:
        for n in ("sw1", "sw3", "sw2"):
            g[n] = np.zeros(getattr(p, n).shape, acc)
        for s in range(p.sw1.shape[0]):
            dxs, d1, d3, d2 = _swiglu_backward(x, p.sw1[s], p.sw3[s], p.sw2[s], dout, acc)
            g["sw1"][s], g["sw3"][s], g["sw2"][s] = d1, d3, d2
            dx += dxs
    g["x"] = dx
    return g
