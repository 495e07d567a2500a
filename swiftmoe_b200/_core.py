"""Shared forward machinery of the drop-in MoE modules.

The forward is the reference's route -> dispatch -> experts -> combine pipeline
(models/ultimate_moe.py:254-342, models/baseline_moe.py:191-213) executed by
libswiftmoe:

* world size 1, no profiling: ONE C-ABI call (``smoe_layer_fwd``) that enqueues the
  router, dispatch plan, permute, grouped expert GEMMs and combine on the current
  stream with no host synchronisation;
* world size 1 with profiling: the same call with the library recording its stage
  events (read lazily in get_profile_summary, no synchronisation inside forward);
* expert parallelism: the kernels called stage by stage around the chunked, overlapped
  all-to-all of ``ep.ExpertParallelExchange``, with CUDA events at the stage boundaries.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from . import _lib as L
from . import kernels as K

STAGES = ("Router", "Dispatch_Comm", "Expert_Compute", "Combine_Comm")
# The reference's profile_data keys (models/ultimate_moe.py:211-216), in STAGES order.
DATA_KEYS = ("router", "dispatch", "compute", "combine")


def resolve_dtype(use_fp16: bool, dtype) -> torch.dtype:
    if dtype is None:
        return torch.float16 if use_fp16 else torch.float32
    if isinstance(dtype, str):
        dtype = {"fp32": torch.float32, "float32": torch.float32, "fp16": torch.float16, "float16": torch.float16,
                 "bf16": torch.bfloat16, "bfloat16": torch.bfloat16}[dtype]
    if dtype not in L.DTYPE_CODE:
        raise ValueError(f"unsupported dtype {dtype}")
    return dtype


def capacity_rows(capacity_factor: Optional[float], tokens_per_rank: int, world_size: int, k: int,
                  num_experts: int) -> int:
    """Per-expert capacity ``ceil(cf * T * ws * k / E)``; 0 means unlimited."""
    if capacity_factor is None:
        return 0
    return int(math.ceil(capacity_factor * tokens_per_rank * world_size * k / num_experts))


def exposed_span(name: str) -> bool:
    """Whether the compute stream is idle for communication from the stage mark ``name``
    to the next mark: the count exchange, a wait on an exchange event ("wait_*_before"),
    or a host wait on the exchange ("host_wait", which also covers the host's
    bookkeeping until the next mark)."""
    return name == "counts_start" or name == "host_wait" or (name.startswith("wait_") and name.endswith("_before"))


class _StageTimer:
    """CUDA-event stage timing without host synchronisation inside forward.

    ``data`` holds, per forward, milliseconds under the reference's keys ``router``,
    ``dispatch``, ``compute`` and ``combine`` (models/ultimate_moe.py:211-216) plus
    ``exposed_a2a``: the time the compute stream sat idle waiting for the exchange."""

    def __init__(self):
        self.pending: List[tuple] = []
        self.data: Dict[str, List[float]] = {s: [] for s in DATA_KEYS}
        self.data["exposed_a2a"] = []
        self.spans: Dict[str, List[float]] = {}   # expert-parallel forward: mark -> next mark

    def mark(self, device) -> torch.cuda.Event:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(device))
        return ev

    def add_marks(self, marks: List[tuple]):
        """(name, event) marks of a stage-by-stage forward (see ep.ExpertParallelExchange)."""
        self.pending.append(("marks", marks))

    def add_library(self, ev: "L.StageEvents"):
        """Events recorded inside smoe_layer_fwd: start, router, dispatch, gemm1, gemm2, combine."""
        self.pending.append(("lib", ev))

    def flush(self):
        for kind, events in self.pending:
            if kind == "marks":
                ev = dict(events)
                events[-1][1].synchronize()
                span = lambda a, b: ev[a].elapsed_time(ev[b])
                names = [n for n, _ in events]
                self.data["router"].append(span("start", "router"))
                self.data["dispatch"].append(span("router", "counts_done"))
                self.data["compute"].append(sum(span(n, n[:-len("_start")] + "_end") for n in names
                                                if n.startswith("experts") and n.endswith("_start")))
                self.data["combine"].append(span("combine_start", "end"))
                self.data["exposed_a2a"].append(sum(ea.elapsed_time(eb) for (a, ea), (_, eb)
                                                    in zip(events[:-1], events[1:]) if exposed_span(a)))
                for (a, ea), (b, eb) in zip(events[:-1], events[1:]):
                    self.spans.setdefault(f"{a}>{b}", []).append(ea.elapsed_time(eb))
                continue
            spans = [(0, 1), (1, 2), (2, 4), (4, 5)]
            for key, (i, j) in zip(DATA_KEYS, spans):
                self.data[key].append(events.elapsed(i, j))
            self.data["exposed_a2a"].append(0.0)
        self.pending.clear()


class _LayerFunction(torch.autograd.Function):
    """The layer as one autograd node: the fused forward, and ``smoe_layer_bwd`` for
    the gradients of x, the gate and every expert weight (16-bit SwiGLU layers on one
    GPU; other layers raise in backward)."""

    @staticmethod
    def forward(ctx, module, x, *params):
        ctx.module = module
        ctx.save_for_backward(x)
        return module._forward_impl(x)

    @staticmethod
    def backward(ctx, dout):
        (x,) = ctx.saved_tensors
        m = ctx.module
        grads = m._backward_fused(x, dout.contiguous())
        return (None, grads["x"] if ctx.needs_input_grad[1] else None, *m._param_grads(grads))


class MoECore(nn.Module):
    """Base class; subclasses provide the parameter accessors."""

    # ---- filled by subclasses
    num_experts: int
    d_model: int
    top_k: int
    expert_type: str
    d_ff: int
    ws: int
    exp_per_rank: int
    capacity_factor: Optional[float]
    num_shared_experts: int
    d_ff_shared: int
    compute_dtype: torch.dtype

    def _init_core(self, enable_profiling: bool):
        self.enable_profiling = enable_profiling
        self._timer = _StageTimer()
        self._ws_buf: Optional[torch.Tensor] = None
        self._wcache: Dict[str, tuple] = {}
        self._soff: Dict[tuple, torch.Tensor] = {}   # shared expert: [0, T] per batch size
        self.comm = None

    # ------------------------------------------------------------ accessors
    def _gate(self) -> torch.Tensor:
        raise NotImplementedError

    def _linear_kmajor(self) -> torch.Tensor:
        """Linear expert weights as [E_l, d_out, d_in] (K contiguous)."""
        raise NotImplementedError

    def _linear_xw(self):
        """Linear expert weights as [E_l, d_in, d_out] (the x @ W layout), and whether the
        module's parameter has that layout (its gradient is then wanted in it too)."""
        raise NotImplementedError

    def _swiglu(self):
        raise NotImplementedError

    def _shared(self):
        return None

    def _logit_bias(self) -> Optional[torch.Tensor]:
        b = getattr(self, "logit_bias", None)
        if b is None:
            return None
        return b.float().contiguous() if (b.dtype != torch.float32 or not b.is_contiguous()) else b

    def _cached(self, key: str, sources: List[torch.Tensor], build):
        sig = tuple((t.data_ptr(), t._version, t.device) for t in sources)
        hit = self._wcache.get(key)
        if hit is not None and hit[0] == sig:
            return hit[1]
        val = build()
        self._wcache[key] = (sig, val)
        return val

    def _workspace(self, nbytes: int, device) -> torch.Tensor:
        if self._ws_buf is None or self._ws_buf.numel() < nbytes or self._ws_buf.device != device:
            self._ws_buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        return self._ws_buf

    # ------------------------------------------------------------ forward
    def _prepare_input(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.d_model:
            raise ValueError(f"expected x of shape [M, {self.d_model}], got {tuple(x.shape)}")
        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        if not x.is_cuda:
            raise L.SwiftMoEError("swiftmoe_b200 runs on CUDA devices only (no CPU fallback); move the module "
                                  "and the input to a GPU")
        return x.contiguous()

    def _capacity(self, T: int) -> int:
        return capacity_rows(self.capacity_factor, T, self.ws, self.top_k, self.num_experts)

    _force_staged = False   # tests: run the stage-by-stage path at world size 1 too

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self._prepare_input(x)
        if torch.is_grad_enabled():
            params = self._grad_params()
            if x.requires_grad or any(p.requires_grad for p in params):
                return _LayerFunction.apply(self, x, *params)
        return self._forward_impl(x)

    def _forward_impl(self, x: torch.Tensor) -> torch.Tensor:
        if self.ws == 1 and not self._force_staged:
            ev = None
            if self.enable_profiling:
                ev = L.StageEvents()
                self._timer.add_library(ev)
            return self._forward_fused(x, ev)
        return self._forward_staged(x)

    def _layer_args(self, x: torch.Tensor, out: torch.Tensor) -> L.LayerArgs:
        a = L.LayerArgs()
        T = x.shape[0]
        a.tokens, a.d_model, a.num_experts, a.top_k = T, self.d_model, self.num_experts, self.top_k
        a.dtype = L.dtype_code(self.compute_dtype)
        # fp32 layers keep their routed expert weights split for the tf32 tensor cores
        # (rebuilt when a weight changes), instead of the library splitting them per call
        split = (self.compute_dtype == torch.float32 and self.d_model % 8 == 0 and
                 (self.expert_type != "swiglu" or self.d_ff % 8 == 0) and
                 os.environ.get("SMOE_FP32_GEMM") != "simt" and os.environ.get("SMOE_FP32_SPLIT_CACHE") != "0")
        if split:
            a.dtype = L.SMOE_F32_SPLITW
        a.capacity = self._capacity(T)
        a.x, a.gate_w, a.out = x.data_ptr(), self._gate().data_ptr(), out.data_ptr()
        bias = self._logit_bias()
        a.logit_bias = bias.data_ptr() if bias is not None else None
        keep = [bias]
        if self.expert_type == "swiglu":
            w1, w3, w2 = self._swiglu()
            if split:
                w1, w3, w2 = (self._cached(name, [w], lambda w=w: K.tf32_split_weights(w.detach()))
                              for name, w in (("w1_tf32", w1), ("w3_tf32", w3), ("w2_tf32", w2)))
            a.expert_type, a.d_ff = L.SMOE_EXPERT_SWIGLU, self.d_ff
            a.w1, a.w3, a.w2 = w1.data_ptr(), w3.data_ptr(), w2.data_ptr()
            keep += [w1, w3, w2]
        else:
            wl = self._linear_kmajor()
            if split:
                wl = self._cached("wl_tf32", [wl], lambda: K.tf32_split_weights(wl.detach()))
            a.expert_type, a.d_ff = L.SMOE_EXPERT_LINEAR, 0
            a.w_lin = wl.data_ptr()
            keep.append(wl)
        sh = self._shared()
        if sh is not None:
            s1, s3, s2 = sh
            a.num_shared, a.d_ff_shared = 1, s1.shape[0]
            a.sw1, a.sw3, a.sw2 = s1.data_ptr(), s3.data_ptr(), s2.data_ptr()
            keep += [s1, s3, s2]
        self._keep_alive = keep
        return a

    def _forward_fused(self, x: torch.Tensor, events: Optional["L.StageEvents"] = None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
        lib = L.load()
        if out is None:
            out = torch.empty_like(x)
        a = self._layer_args(x, out)
        need = lib.smoe_layer_workspace_size(C.byref(a))
        ws = self._workspace(need, x.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        if events is not None:
            events.attach(a)
        L.check(lib.smoe_layer_fwd(C.byref(a), L.stream_handle(x.device)), "smoe_layer_fwd")
        return out

    def _experts(self, xe: torch.Tensor, offsets: torch.Tensor, ends: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, row_ptrs: Optional[torch.Tensor] = None):
        """Expert outputs for the rows of local expert g: [offsets[g], offsets[g+1]), or
        [offsets[g], ends[g]) when ``ends`` is given (other rows are left unwritten).
        The output rows go to ``out`` (same row numbers as ``xe``), or to the addresses in
        ``row_ptrs`` (then None is returned)."""
        if self.expert_type == "swiglu":
            w1, w3, w2 = self._swiglu()
            h = K.grouped_gemm(xe, w1, offsets, B3=w3, epilogue=L.SMOE_EPI_SWIGLU, ends=ends)
            return K.grouped_gemm(h, w2, offsets, ends=ends, out=out, row_ptrs=row_ptrs)
        return K.grouped_gemm(xe, self._linear_kmajor(), offsets, ends=ends, out=out, row_ptrs=row_ptrs)

    def _shared_out(self, x: torch.Tensor) -> Optional[torch.Tensor]:
        sh = self._shared()
        if sh is None:
            return None
        s1, s3, s2 = sh
        T = x.shape[0]
        key = (T, x.device)
        soff = self._soff.get(key)
        if soff is None:    # one group of all T rows; built once per batch size
            soff = self._soff[key] = torch.tensor([0, T], dtype=torch.int32, device=x.device)
        hs = K.grouped_gemm(x, s1.unsqueeze(0), soff, B3=s3.unsqueeze(0), epilogue=L.SMOE_EPI_SWIGLU)
        return K.grouped_gemm(hs, s2.unsqueeze(0), soff)

    def _forward_staged(self, x: torch.Tensor) -> torch.Tensor:
        prof = self.enable_profiling
        dev = x.device
        T = x.shape[0]
        marks = []

        def mark(name):
            if prof:
                marks.append((name, self._timer.mark(dev)))

        mark("start")
        idx, w = K.router(x, self._gate(), self.top_k, self._logit_bias())
        mark("router")
        shared = self._shared_out(x)
        if self.ws == 1:
            plan = K.dispatch_plan(idx, self.num_experts, self._capacity(T))
            xe = K.permute_rows(x, plan["row_token"], plan["offsets"], plan["rows_cap"])
            mark("counts_start")
            mark("counts_done")
            mark("experts0_start")
            y = self._experts(xe, plan["offsets"])
            mark("experts0_end")
            mark("combine_start")
            out = K.combine(y, plan["slot_row"], w, T, self.top_k, shared=shared)
        else:
            out = self.comm.forward(x, idx, w, self._capacity(T), self._experts, shared=shared,
                                    timer=mark if prof else None)
        mark("end")
        if prof:
            self._timer.add_marks(marks)
        return out

    # ------------------------------------------------------------ backward
    def _grad_params(self) -> List[torch.Tensor]:
        """The parameters the layer's autograd node differentiates, in _param_grads order."""
        raise NotImplementedError

    def _param_grads(self, g: Dict[str, torch.Tensor]) -> List[torch.Tensor]:
        """The gradients of _grad_params() from _backward_fused's dict."""
        raise NotImplementedError

    def _backward_ep(self, x: torch.Tensor, dout: torch.Tensor) -> Dict[str, torch.Tensor]:
        """Expert parallelism (world size > 1): ``ep.ExpertParallelExchange.layer_backward``
        with this layer's weights; the same dict as ``_backward_fused``.  The gate's and the
        shared expert's gradients are this rank's contribution (replicated weights); the
        local experts' gradients cover every rank's tokens."""
        if self.comm is None:
            raise NotImplementedError("expert-parallel backward needs the layer's exchange (world size > 1)")
        T = x.shape[0]
        if self.expert_type == "swiglu":
            w1, w3, w2 = self._swiglu()
            F = self.d_ff
            experts = dict(kind="swiglu", w1=w1.detach(), w3=w3.detach(),
                           w2t=self._cached("w2t", [w2], lambda: K.transpose_batched(w2.detach().contiguous())),
                           w13t=self._cached("w13t", [w1, w3], lambda: K.transpose_batched(
                               torch.cat([w1.detach(), w3.detach()], dim=1).contiguous())))
        else:
            wl, xw_layout = self._linear_xw()
            experts = dict(kind="linear", w=wl.contiguous(), transposed=bool(xw_layout))
        sh = None
        if self._shared() is not None:
            s1, s3, s2 = self._shared()
            sh = dict(w1=s1.detach().unsqueeze(0), w3=s3.detach().unsqueeze(0),
                      w2t=self._cached("sw2t", [s2], lambda: K.transpose_batched(s2.detach().unsqueeze(0).contiguous())),
                      w13t=self._cached("sw13t", [s1, s3], lambda: K.transpose_batched(
                          torch.cat([s1.detach(), s3.detach()], dim=0).unsqueeze(0).contiguous())))
        g = self.comm.layer_backward(x.contiguous(), dout.contiguous(), self._gate().detach().contiguous(),
                                     self._logit_bias(), self.top_k, self._capacity(T), experts, sh)
        out = dict(x=g["x"], gate=g["gate"])
        if self.expert_type == "swiglu":
            out.update(w1=g["w13"][:, :F], w3=g["w13"][:, F:], w2=g["w2"])
        else:
            out.update(expert_w=g["lin"])
        if sh is not None:
            Fs = sh["w1"].shape[1]
            out.update(sw1=g["s13"][:Fs], sw3=g["s13"][Fs:], sw2=g["s2"])
        return out

    def _backward_fused(self, x: torch.Tensor, dout: torch.Tensor) -> Dict[str, torch.Tensor]:
        """One ``smoe_layer_bwd`` call: gradients (fp32 for the weights) of the output with
        respect to x ("x", x.dtype), the gate ("gate" [E, d]) and the experts ("w1", "w3"
        [E_l, F, d], "w2" [E_l, d, F]; "sw1", "sw3", "sw2" for the shared expert)."""
        if self.compute_dtype == torch.float32:
            raise NotImplementedError("the backward pass covers 16-bit layers (bf16 / fp16)")
        if self.ws != 1:
            return self._backward_ep(x, dout)
        lib = L.load()
        dev = x.device
        T, d = x.shape
        E = self.num_experts
        a = L.LayerBwdArgs()
        a.tokens, a.d_model, a.num_experts, a.top_k = T, d, E, self.top_k
        a.dtype, a.capacity = L.dtype_code(self.compute_dtype), self._capacity(T)
        f32 = dict(dtype=torch.float32, device=dev)
        dx = torch.empty_like(x)
        dgate = torch.empty((E, d), **f32)
        bias = self._logit_bias()
        keep = [bias]
        a.x, a.dout, a.gate_w = x.data_ptr(), dout.data_ptr(), self._gate().data_ptr()
        a.logit_bias = bias.data_ptr() if bias is not None else None
        a.dx, a.dgate = dx.data_ptr(), dgate.data_ptr()
        out = dict(x=dx, gate=dgate)
        if self.expert_type == "swiglu":
            F = self.d_ff
            w1, w3, w2 = self._swiglu()
            w2t = self._cached("w2t", [w2], lambda: K.transpose_batched(w2.detach().contiguous()))
            w13t = self._cached("w13t", [w1, w3], lambda: K.transpose_batched(
                torch.cat([w1.detach(), w3.detach()], dim=1).contiguous()))
            dw13 = torch.empty((E, 2 * F, d), **f32)
            dw2 = torch.empty((E, d, F), **f32)
            keep += [w2t, w13t]
            a.expert_type, a.d_ff = L.SMOE_EXPERT_SWIGLU, F
            a.w1, a.w3, a.w2t, a.w13t = w1.data_ptr(), w3.data_ptr(), w2t.data_ptr(), w13t.data_ptr()
            a.dw13, a.dw2 = dw13.data_ptr(), dw2.data_ptr()
            out.update(w1=dw13[:, :F], w3=dw13[:, F:], w2=dw2)
        else:
            wlt, xw_layout = self._linear_xw()          # [E, d_in, d_out]
            dwl = torch.empty((E, d, d), **f32)
            keep.append(wlt)
            a.expert_type, a.w_lin_t, a.dw_lin = L.SMOE_EXPERT_LINEAR, wlt.data_ptr(), dwl.data_ptr()
            a.dw_lin_transposed = 1 if xw_layout else 0
            out.update(expert_w=dwl)
        sh = self._shared()
        if sh is not None:
            s1, s3, s2 = sh
            Fs = s1.shape[0]
            s2t = self._cached("sw2t", [s2], lambda: K.transpose_batched(s2.detach().unsqueeze(0).contiguous()))
            s13t = self._cached("sw13t", [s1, s3], lambda: K.transpose_batched(
                torch.cat([s1.detach(), s3.detach()], dim=0).unsqueeze(0).contiguous()))
            dsw13 = torch.empty((2 * Fs, d), **f32)
            dsw2 = torch.empty((d, Fs), **f32)
            a.num_shared, a.d_ff_shared = 1, Fs
            a.sw1, a.sw3, a.sw2t, a.sw13t = s1.data_ptr(), s3.data_ptr(), s2t.data_ptr(), s13t.data_ptr()
            a.dsw13, a.dsw2 = dsw13.data_ptr(), dsw2.data_ptr()
            keep += [s2t, s13t]
            out.update(sw1=dsw13[:Fs], sw3=dsw13[Fs:], sw2=dsw2)
        need = lib.smoe_layer_bwd_workspace_size(C.byref(a))
        wsb = torch.empty(max(int(need), 1), dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = wsb.data_ptr(), wsb.numel()
        L.check(lib.smoe_layer_bwd(C.byref(a), L.stream_handle(dev)), "smoe_layer_bwd")
        return out

    # ------------------------------------------------------------ profiling API
    def get_profile_summary(self) -> Dict[str, float]:
        """Mean milliseconds per stage under the reference's summary keys
        (models/ultimate_moe.py:344-352), plus ``Exposed_A2A``: the mean time per forward
        the compute stream waited for the expert-parallel exchange (counted from the
        stage marks, including host waits; 0 at world size 1)."""
        self._timer.flush()
        mean = lambda v: float(sum(v) / len(v)) if v else 0.0
        out = {name: mean(self._timer.data[key]) for name, key in zip(STAGES, DATA_KEYS)}
        out["Exposed_A2A"] = mean(self._timer.data["exposed_a2a"])
        return out

    def get_profile_spans(self) -> Dict[str, float]:
        """Expert-parallel forwards: mean milliseconds between consecutive stage marks on
        the compute stream (keys "mark>next_mark"), in timeline order."""
        self._timer.flush()
        return {k_: float(sum(v) / len(v)) for k_, v in self._timer.spans.items() if v}

    def reset_profiling(self):
        """models/ultimate_moe.py:354-357."""
        self._timer.flush()
        for v in self._timer.data.values():
            v.clear()
        self._timer.spans.clear()

    @property
    def profile_data(self) -> Dict[str, List[float]]:
        """Per-forward stage milliseconds under the reference's keys ``router``,
        ``dispatch``, ``compute``, ``combine`` (models/ultimate_moe.py:211-216), plus
        ``exposed_a2a``.  Reading it waits for the recorded forwards to finish."""
        self._timer.flush()
        return self._timer.data
