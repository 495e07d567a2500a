"""Drop-in ``StandardMoE`` / ``BaselineMoE`` (models/baseline_moe.py:12-213 of SwiftMoE).

Keeps the reference constructor, the ``gate`` / ``experts[i]`` ``nn.Linear`` parameters
(so reference state_dicts load unchanged) and the private stage methods
``_route_tokens`` / ``_dispatch_tokens`` / ``_expert_forward`` / ``_combine_tokens``,
which chained as the reference's ``forward`` chains them compute the same output as
``forward`` bit for bit.  ``forward`` runs the fused sm_100a path.  Gate weights are
applied after the expert (post-weighting, models/baseline_moe.py:162).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import kernels as K
from . import stages
from ._core import MoECore, resolve_dtype
from .ep import ExpertParallelExchange


class SwiGLUExpert(nn.Module):
    """Extension expert: ``w2(silu(w1 x) * w3 x)`` with nn.Linear parameters."""

    def __init__(self, d_model: int, d_ff: int, dtype=None, device=None):
        super().__init__()
        self.w1 = nn.Linear(d_model, d_ff, bias=False, dtype=dtype, device=device)
        self.w3 = nn.Linear(d_model, d_ff, bias=False, dtype=dtype, device=device)
        self.w2 = nn.Linear(d_ff, d_model, bias=False, dtype=dtype, device=device)


class StandardMoE(MoECore):
    def __init__(self, num_experts: int = 128, d_model: int = 1024, use_fp16: bool = True,
                 world_size: Optional[int] = None, *, top_k: int = 2, d_ff: Optional[int] = None,
                 expert_type: str = "linear", dtype=None, capacity_factor: Optional[float] = None,
                 num_shared_experts: int = 0, d_ff_shared: Optional[int] = None, device=None,
                 init_std: float = 0.02):
        super().__init__()
        self.num_experts = num_experts
        self.d_model = d_model
        self.use_fp16 = use_fp16
        pg_ws = dist.get_world_size() if dist.is_initialized() else 1
        self.world_size = pg_ws if world_size is None else world_size
        if self.world_size != pg_ws:
            raise ValueError(f"world_size={self.world_size} does not match the process group ({pg_ws})")
        self.ws = self.world_size
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        if num_experts % self.ws:
            raise ValueError("num_experts must be divisible by the world size")
        self.experts_per_rank = self.exp_per_rank = num_experts // self.ws
        self.top_k = top_k
        self.expert_type = expert_type
        self.capacity_factor = capacity_factor
        self.num_shared_experts = num_shared_experts
        self.compute_dtype = resolve_dtype(use_fp16, dtype)
        dt = self.compute_dtype
        self.gate = nn.Linear(d_model, num_experts, bias=False, dtype=dt, device=device)
        if expert_type == "linear":
            self.d_ff = 0
            self.experts = nn.ModuleList([nn.Linear(d_model, d_model, bias=False, dtype=dt, device=device)
                                          for _ in range(self.experts_per_rank)])
        elif expert_type == "swiglu":
            self.d_ff = d_ff or 4 * d_model
            self.experts = nn.ModuleList([SwiGLUExpert(d_model, self.d_ff, dt, device)
                                          for _ in range(self.experts_per_rank)])
        else:
            raise ValueError("expert_type must be 'linear' or 'swiglu'")
        nn.init.normal_(self.gate.weight, std=init_std)
        for p in self.experts.parameters():
            nn.init.normal_(p, std=init_std)
        if num_shared_experts:
            self.d_ff_shared = d_ff_shared or self.d_ff or 4 * d_model
            self.shared_expert = SwiGLUExpert(d_model, self.d_ff_shared, dt, device)
            for p in self.shared_expert.parameters():
                nn.init.normal_(p, std=init_std)
        else:
            self.d_ff_shared = 0
        self.register_buffer("logit_bias", None)
        self._init_core(False)
        if self.ws > 1:
            self.comm = ExpertParallelExchange(num_experts, self.ws, self.rank, d_model)

    def set_logit_bias(self, bias: Optional[torch.Tensor]):
        self.logit_bias = None if bias is None else bias.detach().float().to(self.gate.weight.device).contiguous()

    # autograd: gate, each expert's Linear weights, the shared expert
    def _grad_params(self):
        if self.expert_type == "swiglu":
            ps = [self.gate.weight] + [e.w1.weight for e in self.experts] + [e.w3.weight for e in self.experts] \
                + [e.w2.weight for e in self.experts]
        else:
            ps = [self.gate.weight] + [e.weight for e in self.experts]
        if self.num_shared_experts:
            s = self.shared_expert
            ps += [s.w1.weight, s.w3.weight, s.w2.weight]
        return ps

    def _param_grads(self, g):
        dt = self.compute_dtype
        out = [g["gate"].to(dt)]
        if self.expert_type == "linear":
            out += [g["expert_w"][i].to(dt) for i in range(self.experts_per_rank)]
        for n in (("w1", "w3", "w2") if self.expert_type == "swiglu" else ()):
            out += [g[n][i].to(dt) for i in range(self.experts_per_rank)]
        if self.num_shared_experts:
            out += [g[n].to(dt) for n in ("sw1", "sw3", "sw2")]
        return out

    # accessors: experts are separate nn.Linear modules; the kernels want them stacked
    def _gate(self):
        return self.gate.weight

    def _linear_kmajor(self):
        ws_ = [e.weight for e in self.experts]
        return self._cached("lin", ws_, lambda: torch.stack([w.detach() for w in ws_]).contiguous())

    def _linear_xw(self):
        ws_ = [e.weight for e in self.experts]
        return self._cached("lin_xw", ws_, lambda: K.transpose_batched(
            torch.stack([w.detach() for w in ws_]).contiguous())), False

    def _swiglu(self):
        w1 = [e.w1.weight for e in self.experts]
        w3 = [e.w3.weight for e in self.experts]
        w2 = [e.w2.weight for e in self.experts]
        return (self._cached("w1", w1, lambda: torch.stack([w.detach() for w in w1]).contiguous()),
                self._cached("w3", w3, lambda: torch.stack([w.detach() for w in w3]).contiguous()),
                self._cached("w2", w2, lambda: torch.stack([w.detach() for w in w2]).contiguous()))

    def _shared(self):
        if not self.num_shared_experts:
            return None
        s = self.shared_expert
        return s.w1.weight, s.w3.weight, s.w2.weight

    # ---- the reference's stage methods (models/baseline_moe.py:56-189), chained by
    # forward in the reference (:191-213); see stages.py for their contract
    def _route_tokens(self, x: torch.Tensor):
        """(top-k expert indices [M,k] int64, softmax weights [M,k] float32)."""
        x = self._prepare_input(x)
        idx, w = K.router(x, self._gate(), self.top_k, self._logit_bias())
        return idx.long(), w

    def _dispatch_tokens(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor):
        """(recv_x [R,d] grouped by local expert, recv_idx [R] local expert of each row,
        recv_weights [R,1] float32, send_list, recv_list, state for _combine_tokens)."""
        x = self._prepare_input(x)
        return stages.dispatch(x, indices, weights, self.num_experts, self._capacity(x.shape[0]),
                               self.comm if self.ws > 1 else None, shared=self._shared_out(x))

    def _expert_forward(self, recv_x: torch.Tensor, recv_idx: torch.Tensor, recv_weights: torch.Tensor):
        """Expert outputs times their gate weights (post-weighting, :155-162), float32."""
        return stages.expert_rows(self._experts, self.exp_per_rank, recv_x, recv_idx, recv_weights)

    def _combine_tokens(self, expert_output, send_list, recv_list, reverse_indices, original_batch_size):
        """Back to the source ranks, k slots summed in slot order: [M, d] in x.dtype."""
        return stages.combine(expert_output, reverse_indices, original_batch_size,
                              self.comm if self.ws > 1 else None)


BaselineMoE = StandardMoE
