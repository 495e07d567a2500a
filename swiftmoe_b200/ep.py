"""Expert-parallel token exchange (dispatch / combine all-to-all) over torch.distributed.

Replaces ``MoEAsyncCommHandler`` (models/ultimate_moe.py:104-155) and
``StandardMoE._dispatch_tokens`` / ``_combine_tokens`` (models/baseline_moe.py:69-189).

Experts are split into contiguous blocks: global expert ``e`` lives on rank
``e // E_l`` as local expert ``e % E_l`` (models/ultimate_moe.py:93-96).  Differences
from the reference:

* the send buffer is built in one pass by the dispatch-plan and permute kernels,
  already grouped by (destination rank, local expert, token, slot); no
  ``repeat_interleave`` copy and no argsort;
* gate weights and local expert ids are NOT sent (the reference sends three payloads,
  :139-141): the receiver derives the local expert of every row from the count matrix
  and the weights are applied by the sender's combine;
* one device-to-host copy of the count matrix per forward (the reference does four:
  ``.item()``, two ``.tolist()`` and the per-expert ``.cpu()`` at :130,136-137,231);
* the capacity cut (extension) happens on the receiver in (source rank, token, slot)
  order, and dropped rows travel back as zeros so the sender's combine needs no mask.

``kernels`` is the module of device operations.  Production code uses
``swiftmoe_b200.kernels`` (CUDA); CPU tests substitute a numpy double to exercise the
collective choreography on gloo ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DispatchState:
    plan: dict              # send-side plan over global experts
    regroup: dict           # receive-side expert-major plan
    send_splits: list
    recv_splits: list
    n_send: int
    n_recv: int
    T: int
    k: int


class ExpertParallelExchange:
    def __init__(self, num_experts: int, world_size: int, rank: int, d_model: int,
                 group: Optional[dist.ProcessGroup] = None, kernels=None):
        if num_experts % world_size:
            raise ValueError("num_experts must be divisible by the world size")
        self.num_experts = num_experts
        self.world_size = world_size
        self.rank = rank
        self.d_model = d_model
        self.exp_per_rank = num_experts // world_size
        self.group = group
        if kernels is None:
            from . import kernels as _k
            kernels = _k
        self.k = kernels
        self._host = None

    def _counts_to_host(self, counts: torch.Tensor, recv_counts: torch.Tensor):
        """The one host synchronisation of the forward: both count vectors at once."""
        n = counts.numel()
        if counts.is_cuda:
            if self._host is None or self._host.numel() < 2 * n:
                self._host = torch.empty(2 * n, dtype=torch.int32, pin_memory=True)
            h = self._host
            h[:n].copy_(counts, non_blocking=True)
            h[n:2 * n].copy_(recv_counts, non_blocking=True)
            torch.cuda.current_stream(counts.device).synchronize()
            return h[:n].clone(), h[n:2 * n].clone()
        return counts.clone(), recv_counts.clone()

    def dispatch(self, x: torch.Tensor, idx: torch.Tensor, capacity: int = 0):
        """Send every (token, slot) row to the rank owning its expert.

        Returns (rows grouped by local expert [rows, d], expert offsets [E_l+1], state)."""
        ws, El = self.world_size, self.exp_per_rank
        T, k = idx.shape
        plan = self.k.dispatch_plan(idx, self.num_experts)
        send_rows = self.k.permute_rows(x, plan["row_token"], plan["offsets"], plan["rows_cap"])
        counts = plan["counts"]
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        hc, hr = self._counts_to_host(counts, recv_counts)
        send_splits = [int(v) for v in hc.view(ws, El).sum(1).tolist()]
        recv_splits = [int(v) for v in hr.view(ws, El).sum(1).tolist()]
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        recv_rows = torch.empty((max(n_recv, 1), x.shape[1]), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(recv_rows[:n_recv], send_rows[:n_send], recv_splits, send_splits, group=self.group)
        rg = self.k.ep_regroup_plan(recv_counts.view(ws, El), capacity, n_recv)
        xe = self.k.permute_rows(recv_rows, rg["row_src"], rg["offsets"], rg["rows_cap"])
        st = DispatchState(plan, rg, send_splits, recv_splits, n_send, n_recv, T, k)
        return xe, rg["offsets"], st

    def combine(self, y: torch.Tensor, st: DispatchState, w: torch.Tensor,
                shared: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
        """Return expert outputs to their source ranks and reduce the k slots."""
        back = self.k.gather_rows(y, st.regroup["recv_dst"], st.n_recv)
        ret = torch.empty((max(st.n_send, 1), y.shape[1]), dtype=y.dtype, device=y.device)
        dist.all_to_all_single(ret[:st.n_send], back[:st.n_recv], st.send_splits, st.recv_splits, group=self.group)
        return self.k.combine(ret, st.plan["slot_row"], w, st.T, st.k, shared=shared, out=out)
