"""The reference's stage-by-stage interface over this library's kernels.

The reference splits its layers into stages that callers can run one at a time:
``StandardMoE._route_tokens -> _dispatch_tokens -> _expert_forward -> _combine_tokens``
(models/baseline_moe.py:56-189, chained by its ``forward`` at :191-213) and
``MoEAsyncCommHandler.dispatch -> UltimateMoE._expert_compute ->
MoEAsyncCommHandler.combine`` (models/ultimate_moe.py:104-155, 222-252, 301-338).  The
functions here give those stages the reference's arguments and return values, and
chained in the reference's order they compute exactly what ``forward`` computes:

* routing returns float32 gate weights (the reference returns them in x.dtype): they
  are the weights the fused forward applies;
* dispatch returns the routed rows grouped by local expert, each row's local expert id
  and its gate weight (the reference's ``recv_x, recv_local_idx, recv_weights``), the
  per-rank send / receive counts as lists, and a state object that takes the place of
  the reference's ``reverse_indices``;
* the expert stage weights each output row by its gate weight in float32 (the
  reference multiplies in x.dtype) and returns float32 rows;
* combine returns the rows to their source ranks and sums each token's k slots in slot
  order, in float32 (plus the shared expert's output), rounded once to x.dtype.

Weighted fp32 rows summed in slot order are the same arithmetic as the fused combine
kernel, which rounds each product w * y to fp32 before adding it, so the chain and
``forward`` agree bit for bit.  The stages synchronise with the host where the
reference does (the counts become Python lists); ``forward`` itself never does.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _lib as L
from . import kernels as K


@dataclass
class StageState:
    """What combine needs from dispatch (the reference passes ``reverse_indices``)."""
    slot_row: Optional[torch.Tensor]   # world size 1: slot -> row of the expert-major rows (-1: dropped)
    exchange_state: object             # world size > 1: ep.DispatchState of the exchange
    T: int
    k: int
    dtype: torch.dtype
    shared: Optional[torch.Tensor]     # shared expert output [T, d] (extension), or None


def _row_slots(slot_row: torch.Tensor, n_rows: int) -> torch.Tensor:
    """Inverse of slot_row: the (token, slot) index of every row (-1 for none), without a
    host synchronisation (dropped slots are scattered into a spare last entry)."""
    n_slots = slot_row.numel()
    dev = slot_row.device
    inv = torch.full((n_rows + 1,), -1, dtype=torch.int64, device=dev)
    tgt = torch.where(slot_row >= 0, slot_row.long(), torch.full_like(slot_row, n_rows, dtype=torch.int64))
    inv.scatter_(0, tgt, torch.arange(n_slots, device=dev, dtype=torch.int64))
    return inv[:n_rows]


def _row_weights(w: torch.Tensor, row_slot: torch.Tensor) -> torch.Tensor:
    flat = w.reshape(-1).float()
    return torch.where(row_slot >= 0, flat[row_slot.clamp(min=0)], torch.zeros((), device=w.device))


def _local_ids(offsets: torch.Tensor, n_rows: int) -> torch.Tensor:
    """Local expert of every row of an expert-major layout with group offsets [G+1]."""
    r = torch.arange(n_rows, device=offsets.device, dtype=torch.int32)
    return torch.searchsorted(offsets[1:].contiguous(), r, right=True).to(torch.int32)


def dispatch(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int, capacity: int,
             exchange=None, shared: Optional[torch.Tensor] = None):
    """Routed rows grouped by (local) expert: (rows [R, d], local expert ids [R] int32,
    gate weights [R, 1] fp32, send list, receive list, StageState).  ``exchange`` is the
    layer's ep.ExpertParallelExchange at world size > 1, else None."""
    T, k = idx.shape
    idx = idx.to(torch.int32).contiguous()
    w = w.float().contiguous()
    if exchange is None:
        plan = K.dispatch_plan(idx, num_experts, capacity)
        n = int(plan["offsets"][num_experts])           # the reference's .tolist() sync
        rows = K.permute_rows(x, plan["row_token"], plan["offsets"], plan["rows_cap"])[:n]
        ids = _local_ids(plan["offsets"], n)
        rw = _row_weights(w, _row_slots(plan["slot_row"], plan["rows_cap"]))[:n]
        st = StageState(plan["slot_row"], None, T, k, x.dtype, shared)
        return rows, ids, rw.view(-1, 1), [n], [n], st
    rows, offsets, xst, rw = exchange.dispatch(x, idx, capacity, slot_payload=w)
    El = exchange.exp_per_rank
    n = int(offsets[El])
    ids = _local_ids(offsets, n)
    st = StageState(None, xst, T, k, x.dtype, shared)
    return rows[:n], ids, rw[:n].view(-1, 1), list(xst.send_splits), list(xst.recv_splits), st


def expert_rows(experts, num_local: int, recv_x: torch.Tensor, recv_idx: torch.Tensor,
                recv_w: torch.Tensor) -> torch.Tensor:
    """Expert outputs of the received rows weighted by their gate weights, in float32, in
    the order of ``recv_x`` (any order; rows whose expert id is outside [0, num_local)
    give zero rows).  ``experts(rows, offsets)`` runs the grouped expert GEMMs."""
    n, d = recv_x.shape
    dev = recv_x.device
    if n == 0:
        return torch.zeros((0, d), dtype=torch.float32, device=dev)
    ids = recv_idx.reshape(-1).to(torch.int32)
    valid = (ids >= 0) & (ids < num_local)
    key = torch.where(valid, ids, torch.full_like(ids, num_local))
    order = torch.sort(key, stable=True).indices.to(torch.int32)          # grouped by expert
    xs = K.gather_rows(recv_x.contiguous(), order.contiguous(), n)
    offsets = torch.searchsorted(key[order.long()].contiguous(),
                                 torch.arange(num_local + 1, device=dev, dtype=torch.int32)).to(torch.int32)
    y = experts(xs, offsets)[:n]
    wz = recv_w.reshape(-1).float()[order.long()]
    z = torch.where(valid[order.long()].view(-1, 1), y.float() * wz.view(-1, 1), torch.zeros((), device=dev))
    out = torch.empty((n, d), dtype=torch.float32, device=dev)
    out[order.long()] = z
    return out


def combine(expert_out: torch.Tensor, st: StageState, M: int, exchange=None) -> torch.Tensor:
    """Sum of each token's k weighted slot rows (slot order, fp32) plus the shared
    expert, rounded to the dispatched dtype: [M, d]."""
    if M != st.T:
        raise L.SwiftMoEError(f"combine for {M} tokens, but {st.T} were dispatched")
    y = expert_out if expert_out.dtype == torch.float32 else expert_out.float()
    y = y.contiguous()
    dev = y.device
    ones = torch.ones((st.T, st.k), dtype=torch.float32, device=dev)
    shared = None if st.shared is None else st.shared.float().contiguous()
    if st.exchange_state is None:
        if y.shape[0] == 0:
            y = torch.zeros((1, y.shape[1]), dtype=torch.float32, device=dev)
        out = K.combine(y, st.slot_row, ones, st.T, st.k, shared=shared)
    else:
        out = exchange.combine(y, st.exchange_state, ones, shared=shared)
    return out.to(st.dtype)


class MoEAsyncCommHandler:
    """The reference's exchange object (models/ultimate_moe.py:104-155) with its
    constructor and methods:

        comm = MoEAsyncCommHandler(num_experts, world_size, d_model, device)
        recv_x, recv_local_idx, recv_w, s_list, r_list, rev = comm.dispatch(
            x, indices, weights, target_ranks, local_indices)
        out = comm.combine(expert_out, s_list, r_list, rev, M)

    ``target_ranks`` / ``local_indices`` are accepted for the signature and not needed
    (both follow from ``indices``: experts are split in contiguous blocks).  Received
    rows come grouped by local expert rather than by source rank; ``rev`` is this
    library's dispatch state.  ``combine`` sums the k slots of each token in slot order
    (the reference's ``view(M, 2, d).sum(1)`` for k = 2), in float32, returning x.dtype.
    At world size > 1 a process group must exist; the payload goes through the
    collective transport of ep.ExpertParallelExchange."""

    def __init__(self, num_experts, world_size, d_model, device, *, capacity: int = 0, group=None):
        from .ep import ExpertParallelExchange
        if num_experts % world_size:
            raise ValueError("num_experts must be divisible by the world size")
        self.num_experts = num_experts
        self.world_size = world_size
        self.d_model = d_model
        self.device = torch.device(device)
        self.exp_per_rank = num_experts // world_size
        self.capacity = capacity
        self._exchange = None
        if world_size > 1:
            rank = dist.get_rank(group) if dist.is_initialized() else 0
            self._exchange = ExpertParallelExchange(num_experts, world_size, rank, d_model, group=group,
                                                    transport="collective")

    def dispatch(self, x, indices, weights, target_ranks=None, local_indices=None):
        if not x.is_cuda:
            raise L.SwiftMoEError("swiftmoe_b200 runs on CUDA devices only (no CPU fallback)")
        idx = indices.reshape(x.shape[0], -1)
        w = weights.reshape(x.shape[0], -1)
        return dispatch(x.contiguous(), idx, w, self.num_experts, self.capacity, self._exchange)

    def combine(self, expert_out, s_list, r_list, sort_idx_rev, M):
        return combine(expert_out, sort_idx_rev, M, self._exchange)
