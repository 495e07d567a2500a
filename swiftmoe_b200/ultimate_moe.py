"""Drop-in ``UltimateMoE`` (models/ultimate_moe.py:158-357 of SwiftMoE) on sm_100a kernels.

Same constructor prefix, attributes, parameter names/layouts and ``forward(x[M, d])``;
keyword-only extensions add SwiGLU experts, top-k != 2, bf16, capacity dropping, an
always-on shared expert and per-expert router logit offsets.  ``use_triton`` is
accepted for signature compatibility and has no effect (there is no Triton here).
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import kernels as K
from . import stages
from ._core import MoECore, resolve_dtype
from .ep import ExpertParallelExchange


def setup_nccl_optimizations():
    """The reference's NCCL settings (models/ultimate_moe.py:15-31), with one left out.

    Same values as the reference for NCCL_IB_DISABLE, NCCL_P2P_LEVEL,
    NCCL_NET_GDR_LEVEL, NCCL_MIN_NCHANNELS, NCCL_BUFFSIZE and NCCL_NTHREADS.
    NCCL_SOCKET_IFNAME=eth0 is not set: it names a host interface, and on a machine
    whose interface has another name NCCL's bootstrap cannot find it and the group fails
    to form; NCCL's own interface choice works on every host.

    Only variables that are not already set are written.  They take effect for process
    groups created AFTER this call (the reference calls it from the layer constructor,
    after the group exists, where it has no effect); ``init_expert_parallel`` applies
    them before it creates the group."""
    nccl_config = {
        "NCCL_IB_DISABLE": "0",
        "NCCL_P2P_LEVEL": "NVL",
        "NCCL_NET_GDR_LEVEL": "5",
        "NCCL_MIN_NCHANNELS": "12",
        "NCCL_BUFFSIZE": "4194304",
        "NCCL_NTHREADS": "512",
    }
    for key, value in nccl_config.items():
        if key not in os.environ:
            os.environ[key] = value
    return nccl_config


class UltimateMoE(MoECore):
    def __init__(self, num_experts: int = 128, d_model: int = 1024, use_fp16: bool = True, use_triton: bool = True,
                 use_nccl_opt: bool = True, enable_profiling: bool = False, *, top_k: int = 2,
                 d_ff: Optional[int] = None, expert_type: str = "linear", dtype=None,
                 capacity_factor: Optional[float] = None, num_shared_experts: int = 0,
                 d_ff_shared: Optional[int] = None, device=None, init_std: float = 0.02):
        super().__init__()
        self.rank = int(os.environ.get("LOCAL_RANK", 0))
        self.ws = dist.get_world_size() if dist.is_initialized() else 1
        self.num_experts = num_experts
        self.d_model = d_model
        self.use_fp16 = use_fp16
        self.use_triton = use_triton
        self.use_nccl_opt = use_nccl_opt
        if num_experts % self.ws:
            raise ValueError(f"num_experts={num_experts} is not divisible by world size {self.ws}")
        if not 1 <= top_k <= min(num_experts, 32):
            raise ValueError("top_k must be in [1, min(num_experts, 32)]")
        if expert_type not in ("linear", "swiglu"):
            raise ValueError("expert_type must be 'linear' or 'swiglu'")
        if num_shared_experts not in (0, 1):
            raise ValueError("num_shared_experts must be 0 or 1")
        self.exp_per_rank = num_experts // self.ws
        self.top_k = top_k
        self.expert_type = expert_type
        self.capacity_factor = capacity_factor
        self.num_shared_experts = num_shared_experts
        self.compute_dtype = resolve_dtype(use_fp16, dtype)
        dt, El, d = self.compute_dtype, self.exp_per_rank, d_model

        def param(*shape):
            p = nn.Parameter(torch.empty(*shape, dtype=dt, device=device))
            nn.init.normal_(p, std=init_std)
            return p

        if expert_type == "linear":
            self.d_ff = 0
            self.expert_weights = param(El, d, d)           # used as x @ W (reference layout)
        else:
            self.d_ff = d_ff or 4 * d
            self.w1 = param(El, self.d_ff, d)              # gate projection, nn.Linear layout
            self.w3 = param(El, self.d_ff, d)              # up projection
            self.w2 = param(El, d, self.d_ff)              # down projection
        self.gate_weight = param(num_experts, d)
        if num_shared_experts:
            self.d_ff_shared = d_ff_shared or self.d_ff or 4 * d
            self.shared_w1 = param(self.d_ff_shared, d)
            self.shared_w3 = param(self.d_ff_shared, d)
            self.shared_w2 = param(d, self.d_ff_shared)
        else:
            self.d_ff_shared = 0
        self.register_buffer("logit_bias", None)
        self._init_core(enable_profiling)
        if self.ws > 1:
            self.comm = ExpertParallelExchange(num_experts, self.ws, dist.get_rank(), d_model)
        self.compute_stream = None
        if use_nccl_opt:
            setup_nccl_optimizations()

    def set_logit_bias(self, bias: Optional[torch.Tensor]):
        """Per-expert offsets added to the router logits before top-k (extension)."""
        self.logit_bias = None if bias is None else bias.detach().float().to(self.gate_weight.device).contiguous()

    def _expert_compute(self, recv_x: torch.Tensor, recv_idx: torch.Tensor, recv_w: torch.Tensor):
        """Expert stage of the reference's forward (models/ultimate_moe.py:222-252): the
        received rows (any order) through their local experts, each weighted by its gate
        weight.  The weight scales the expert's output in float32 (the reference scales
        its input, which is the same for a linear expert up to rounding), and the rows
        come back in float32 so that MoEAsyncCommHandler.combine rounds once."""
        return stages.expert_rows(self._experts, self.exp_per_rank, recv_x, recv_idx, recv_w)

    # autograd: gate, the expert weights, the shared expert
    def _grad_params(self):
        ps = [self.gate_weight] + ([self.w1, self.w3, self.w2] if self.expert_type == "swiglu"
                                   else [self.expert_weights])
        if self.num_shared_experts:
            ps += [self.shared_w1, self.shared_w3, self.shared_w2]
        return ps

    def _param_grads(self, g):
        out = [g["gate"].to(self.gate_weight.dtype)]
        if self.expert_type == "swiglu":
            out += [g[n].to(self.compute_dtype) for n in ("w1", "w3", "w2")]
        else:
            out.append(g["expert_w"].to(self.compute_dtype))
        if self.num_shared_experts:
            out += [g[n].to(self.compute_dtype) for n in ("sw1", "sw3", "sw2")]
        return out

    # accessors
    def _gate(self):
        return self.gate_weight

    def _linear_kmajor(self):
        w = self.expert_weights
        return self._cached("lin", [w], lambda: K.transpose_batched(w.detach().contiguous()))

    def _linear_xw(self):
        return self.expert_weights.detach(), True

    def _swiglu(self):
        return self.w1, self.w3, self.w2

    def _shared(self):
        if not self.num_shared_experts:
            return None
        return self.shared_w1, self.shared_w3, self.shared_w2


# The reference's exchange class, with its constructor and dispatch / combine signatures.
MoEAsyncCommHandler = stages.MoEAsyncCommHandler
