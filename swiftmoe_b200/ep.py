"""Expert-parallel token exchange (dispatch / combine all-to-all) over torch.distributed,
overlapped with the expert GEMMs.

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
* ONE device-to-host copy of the count matrix per forward (the reference makes four:
  ``.item()``, two ``.tolist()`` and the per-expert ``.cpu()`` at :130,136-137,231);
* on CUDA devices rows move by device-to-device copies into the peers' buffers (copy
  engines over NVLink, CUDA IPC), and the GEMMs of the rows a rank routes to its own
  experts run while the other ranks' rows are in flight ("local first"); the
  alternative schedules send the batch in token chunks on a communication stream, the
  dispatch of chunk c+1 and the return of chunk c-1 running while the expert GEMMs of
  chunk c run on the compute stream (``schedule="chunked"``, and the collective
  transport);
* the capacity cut (extension) happens on the receiver in (source rank, token, slot)
  order over the whole batch, and dropped rows travel back as zeros so the sender's
  combine needs no mask.

``kernels`` is the module of device operations.  Production code uses
``swiftmoe_b200.kernels`` (CUDA); CPU tests substitute a numpy double to exercise the
collective choreography on gloo ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib as L


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


def chunk_bounds(T: int, chunks: int) -> List[tuple]:
    """``chunks`` token ranges covering [0, T), some empty when T < chunks.  The count is
    the same on every rank whatever its batch size, because the ranks exchange one count
    vector per chunk."""
    c = max(1, chunks)
    edges = [T * i // c for i in range(c + 1)]
    return [(edges[i], edges[i + 1]) for i in range(c)]


def capacity_positions(recv_counts: np.ndarray, capacity: int):
    """recv_counts [C, ws, E_l] (chunk, source rank, local expert) -> position base
    [C, ws, E_l]: where each (chunk, source) segment starts in its expert's global
    (source rank, token, slot) order.  Chunks are token ranges of one source, so the
    order is source-major, then chunk."""
    C, ws, El = recv_counts.shape
    per_src = recv_counts.sum(0)                        # [ws, E_l]
    src_start = np.cumsum(per_src, 0) - per_src         # rows of earlier sources
    chunk_start = np.cumsum(recv_counts, 0) - recv_counts
    return (src_start[None] + chunk_start).astype(np.int32)


def kept_rows(rows_per_expert: np.ndarray, capacity: int) -> int:
    """Rows an expert computes after the capacity cut (all of them without a capacity)."""
    r = np.asarray(rows_per_expert, dtype=np.int64)
    return int(np.minimum(r, capacity).sum() if capacity > 0 else r.sum())


class ExpertParallelExchange:
    def __init__(self, num_experts: int, world_size: int, rank: int, d_model: int,
                 group: Optional[dist.ProcessGroup] = None, kernels=None, chunks: int = 4,
                 transport: str = "auto", schedule: str = "device",
                 runtime=None):
        if num_experts % world_size:
            raise ValueError("num_experts must be divisible by the world size")
        self.num_experts = num_experts
        self.world_size = world_size
        self.rank = rank
        self.d_model = d_model
        self.exp_per_rank = num_experts // world_size
        self.group = group
        self.chunks = chunks
        if kernels is None:
            from . import kernels as _k
            kernels = _k
        self.k = kernels
        self._host = None
        self._seg_host = None       # return-address table of the fused return (pinned)
        self._comm_stream = {}
        self._last_rows, self._rows_dev = 0, None   # expert rows of the last forward (last_rows)
        self._ones = None           # unit weights of the dedup path's final combine
        if transport not in ("auto", "p2p", "collective"):
            raise ValueError("transport must be 'auto', 'p2p' or 'collective'")
        self.transport = transport
        self._bufs = None           # (receive, return) PeerBuffers of the p2p transport
        if schedule not in ("device", "local_first", "chunked"):
            raise ValueError("schedule must be 'device', 'local_first' or 'chunked'")
        # p2p transport: "device" (layout on the device, rows stored into the peers by the
        # send kernel, no host wait), "local_first" (host-computed layout, copy engines)
        # or "chunked" (chunk-by-chunk overlap)
        self.schedule = schedule
        # device schedule: tokens any rank may pass to forward; sizes the peer buffers.
        # None: the largest batch of the first device-schedule forward (one collective).
        self.max_tokens: Optional[int] = None
        self._dev = None            # device schedule: persistent layout tensors
        # local-first return of the other ranks' rows: "fused" = the expert GEMM stores
        # them into the source ranks' buffers; "copy" = gather + device-to-device copies
        self.return_mode = "fused"
        # from this many ranks on, the own rows are computed in two halves (local first)
        self.split_min_ws = 4
        # token dedup on the local-first schedule without capacity: "auto", "on", "off"
        self.dedup = "auto"
        if runtime is None:
            from .p2p import CudaRuntime
            runtime = CudaRuntime()
        self.rt = runtime           # streams, events, peer buffers and copies (p2p transport)
        self._flag = None

    # ------------------------------------------------------------------ helpers
    def _stream(self, device):
        if device.type != "cuda":
            return None
        s = self._comm_stream.get(device.index)
        if s is None:
            s = self._comm_stream[device.index] = torch.cuda.Stream(device)
        return s

    def _to_host(self, *ts):
        """The one host synchronisation of the forward: all count vectors at once."""
        n = sum(t.numel() for t in ts)
        if ts[0].is_cuda:
            if self._host is None or self._host.numel() < n:
                self._host = torch.empty(n, dtype=torch.int32, pin_memory=True)
            h, o = self._host, 0
            for t in ts:
                h[o:o + t.numel()].copy_(t.reshape(-1), non_blocking=True)
                o += t.numel()
            torch.cuda.current_stream(ts[0].device).synchronize()
            out, o = [], 0
            for t in ts:
                out.append(h[o:o + t.numel()].clone().numpy().reshape(t.shape))
                o += t.numel()
            return out
        return [t.numpy().copy() for t in ts]

    def _use_dedup(self, k: int) -> bool:
        """Token dedup pays when a token's k slots often share a rank: "auto" = from k = 4
        on (with k = 2 and one expert per rank nothing repeats, and the receiver's extra
        permute would only cost)."""
        if self.dedup == "auto":
            return k >= 4 and self.exp_per_rank > 1
        return self.dedup == "on"

    @property
    def last_rows(self) -> int:
        """Expert rows (routed slots after the capacity cut) this rank computed in the last
        forward; reading it after a dedup forward synchronises with the device."""
        if self._rows_dev is not None:
            self._last_rows = int(sum(int(t[0]) for t in self._rows_dev))
            self._rows_dev = None
        return self._last_rows

    @last_rows.setter
    def last_rows(self, v: int):
        self._last_rows, self._rows_dev = int(v), None

    def describe(self) -> str:
        """The exchange configuration in words (benchmark records)."""
        if self.transport == "collective":
            return f"collective transport (all_to_all_single), {self.chunks} token chunks"
        if self.schedule == "chunked":
            return f"{self.transport} transport, chunked schedule, {self.chunks} token chunks"
        if self.schedule == "device":
            return (f"{self.transport} transport, device schedule (layout on the device, rows stored into "
                    f"the peers by the send kernel, fused return, no host wait), token dedup {self.dedup} "
                    f"(dedup forwards with k a multiple of 4 on the device schedule too, others on the host-laid-out "
                    f"one), max {self.max_tokens} tokens per rank")
        return (f"{self.transport} transport, local_first schedule, {self.return_mode} return, "
                f"token dedup {self.dedup}, own rows split from {self.split_min_ws} ranks")

    def n_chunks(self, T: int) -> int:
        """Token chunks of the chunked schedules: the same on every rank (the ranks'
        batches may differ in size), so it does not depend on T."""
        return max(1, self.chunks)

    # ------------------------------------------------------------------ the layer
    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, capacity: int,
                experts: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
                shared: Optional[torch.Tensor] = None, timer=None) -> torch.Tensor:
        """Dispatch, expert compute (``experts(rows, offsets)``) and combine for one batch.

        CUDA tensors use the peer-copy transport (``_forward_p2p``) unless
        ``transport="collective"``; CPU tensors (gloo) use all_to_all_single."""
        use_p2p = self.transport == "p2p" or (self.transport == "auto" and x.is_cuda)
        dedup = capacity <= 0 and self._use_dedup(idx.shape[1])
        if use_p2p and self.schedule == "device" and dedup and (idx.shape[1] * 4) % 16 == 0:
            return self._forward_p2p_device_dedup(x, idx, w, experts, shared, timer)
        if use_p2p and self.schedule in ("device", "local_first") and dedup:
            return self._forward_p2p_dedup(x, idx, w, experts, shared, timer)
        if use_p2p and self.schedule == "device":
            return self._forward_p2p_device(x, idx, w, capacity, experts, shared, timer)
        if use_p2p and self.schedule == "local_first":
            return self._forward_p2p_local_first(x, idx, w, capacity, experts, shared, timer)
        if use_p2p:
            return self._forward_p2p(x, idx, w, capacity, experts, shared, timer)
        return self._forward_collective(x, idx, w, capacity, experts, shared, timer)

    def _forward_collective(self, x, idx, w, capacity, experts, shared=None, timer=None):
        """Payload exchange through ``all_to_all_single`` (NCCL or gloo).

        ``timer`` (optional) is called with a stage-boundary name at points of the compute
        stream's timeline; the profiler records an event there.  The spans between
        ``wait_*_before`` and ``wait_*_after`` are the time the compute stream stalls on
        communication, i.e. the exposed all-to-all time."""
        ws, El, E = self.world_size, self.exp_per_rank, self.num_experts
        T, k = idx.shape
        d = x.shape[1]
        dev = x.device
        bounds = chunk_bounds(T, self.n_chunks(T))
        C = len(bounds)
        comp = torch.cuda.current_stream(dev) if dev.type == "cuda" else None
        comm = self._stream(dev)

        def mark(name):
            if timer is not None:
                timer(name)

        # per-chunk send plans and send buffers (compute stream)
        plans, sends = [], []
        for (a, b) in bounds:
            p = self.k.dispatch_plan(idx[a:b], E)
            plans.append(p)
            sends.append(self.k.permute_rows(x[a:b], p["row_token"], p["offsets"], p["rows_cap"]))
        counts = torch.stack([p["counts"] for p in plans]).view(C, ws, El)        # [C, dst, El]
        send_counts = counts.transpose(0, 1).contiguous()                           # [dst, C, El]
        recv_counts = torch.empty_like(send_counts)                                 # [src, C, El]
        mark("counts_start")
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        hc, hr = self._to_host(send_counts, recv_counts)
        mark("counts_done")
        hr_c = np.ascontiguousarray(hr.transpose(1, 0, 2))                          # [C, src, El]
        pos = capacity_positions(hr_c, capacity) if capacity > 0 else None
        pos_dev = None
        if pos is not None:
            pos_dev = torch.from_numpy(pos).to(dev, non_blocking=True)

        send_splits = [[int(v) for v in hc[:, c, :].sum(1)] for c in range(C)]
        recv_splits = [[int(v) for v in hr[:, c, :].sum(1)] for c in range(C)]
        # every buffer another stream writes is allocated here, before that stream waits for
        # the compute stream: a block allocated later could still be read by compute work
        # queued earlier (the caching allocator only orders reuse within one stream)
        recv_rows = [torch.empty((max(sum(recv_splits[c]), 1), d), dtype=x.dtype, device=dev) for c in range(C)]
        rets = [torch.empty((max(sum(send_splits[c]), 1), d), dtype=x.dtype, device=dev) for c in range(C)]
        ev_sent = []
        # dispatch all-to-alls on the communication stream
        if comm is not None:
            comm.wait_stream(comp)
        for c in range(C):
            with _maybe_stream(comm):
                dist.all_to_all_single(recv_rows[c][:sum(recv_splits[c])], sends[c][:sum(send_splits[c])],
                                       recv_splits[c], send_splits[c], group=self.group)
                ev_sent.append(_record(comm))
        # expert compute per chunk as its rows arrive (compute stream)
        backs, states, ev_back = [], [], []
        for c in range(C):
            mark(f"wait_sent{c}_before")
            _wait(comp, ev_sent[c])
            mark(f"wait_sent{c}_after")
            n_recv = sum(recv_splits[c])
            rg = self.k.ep_regroup_plan(recv_counts[:, c, :].contiguous(), capacity, n_recv,
                                        pos_base=None if pos_dev is None else pos_dev[c])
            xe = self.k.permute_rows(recv_rows[c], rg["row_src"], rg["offsets"], rg["rows_cap"])
            mark(f"experts{c}_start")
            y = experts(xe, rg["offsets"])
            mark(f"experts{c}_end")
            backs.append(self.k.gather_rows(y, rg["recv_dst"], n_recv))
            ev_back.append(_record(comp))
            states.append((rg, n_recv))
        self.last_rows = kept_rows(hr.sum((0, 1)), capacity)
        # return all-to-alls (communication stream) and combine (compute stream)
        ev_ret = []
        for c in range(C):
            _wait(comm, ev_back[c])
            with _maybe_stream(comm):
                dist.all_to_all_single(rets[c][:sum(send_splits[c])], backs[c][:states[c][1]],
                                       send_splits[c], recv_splits[c], group=self.group)
                ev_ret.append(_record(comm))
        out = torch.empty_like(x)
        mark("combine_start")
        for c, (a, b) in enumerate(bounds):
            mark(f"wait_ret{c}_before")
            _wait(comp, ev_ret[c])
            mark(f"wait_ret{c}_after")
            self.k.combine(rets[c], plans[c]["slot_row"], w[a:b], b - a, k,
                           shared=None if shared is None else shared[a:b], out=out[a:b])
        return out


    # ------------------------------------------------------------------ peer copies
    def _barrier(self, stream, dev):
        """Orders this rank's copies issued on `stream` before every rank's next work on
        its own `stream`: a one-int all-reduce, which on each rank starts only after that
        rank's earlier copies completed."""
        if self._flag is None or self._flag.device != dev:
            self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
        with self.rt.on(stream):
            dist.all_reduce(self._flag, group=self.group)

    def _peer_buffers(self, dev):
        if self._bufs is None:
            self._bufs = (self.rt.buffers(self.group, self.rank, self.world_size, dev),
                          self.rt.buffers(self.group, self.rank, self.world_size, dev))
        return self._bufs

    def _forward_p2p(self, x, idx, w, capacity, experts, shared=None, timer=None):
        """Chunked schedule: rows travel by device-to-device copies into the peers'
        receive / return buffers (copy engines over NVLink), chunk by chunk on the
        communication stream, while the compute stream runs the expert GEMMs of the
        chunks that have arrived."""
        rt = self.rt
        ws, El, E, me = self.world_size, self.exp_per_rank, self.num_experts, self.rank
        T, k = idx.shape
        d = x.shape[1]
        dev = x.device
        rb = d * x.element_size()
        bounds = chunk_bounds(T, self.n_chunks(T))
        C = len(bounds)
        comp, comm = rt.compute(dev), rt.comm(dev)
        recv_buf, ret_buf = self._peer_buffers(dev)

        def mark(name):
            if timer is not None:
                timer(name)

        plans, sends = [], []
        for (a, b) in bounds:
            p = self.k.dispatch_plan(idx[a:b], E)
            plans.append(p)
            sends.append(self.k.permute_rows(x[a:b], p["row_token"], p["offsets"], p["rows_cap"]))
        counts = torch.stack([p["counts"] for p in plans])                 # [C, E]
        G = torch.empty((ws, C, E), dtype=torch.int32, device=dev)          # [src, C, dst*El]
        mark("counts_start")
        # the count exchange also orders this step after every rank finished reading its
        # buffers in the previous step (each rank joins it after its earlier work)
        dist.all_gather_into_tensor(G.view(-1), counts.reshape(-1), group=self.group)
        (Gh,) = self._to_host(G)
        mark("counts_done")
        Gh = Gh.reshape(ws, C, ws, El).astype(np.int64)
        R = Gh.sum(3)                                   # [src, C, dst] rows src -> dst in chunk c
        recv_c = R.sum(0)                               # [C, dst]
        RO = np.cumsum(recv_c, 0) - recv_c              # chunk region start in dst's receive buffer
        SO = np.cumsum(R, 0) - R                        # src offset inside dst's chunk region
        send_c = R.sum(2)                               # [src, C]
        SRO = np.cumsum(send_c, 1) - send_c             # chunk region start in src's return buffer
        SD = np.cumsum(R, 2) - R                        # dst segment offset inside src's chunk region
        recv_buf.ensure(int(max(recv_c.sum(0).max(), 1)) * rb)
        ret_buf.ensure(int(max(send_c.sum(1).max(), 1)) * rb)
        rc_me = G[:, :, me * El:(me + 1) * El]          # [src, C, El] received by me (device)
        pos_dev = None
        if capacity > 0:
            pos = capacity_positions(np.ascontiguousarray(Gh[:, :, me, :].transpose(1, 0, 2)), capacity)
            pos_dev = torch.from_numpy(pos).to(dev, non_blocking=True)

        rt.join(comm, comp)
        ev_sent = []
        for c in range(C):
            rt.keep(sends[c], comm)
            base = sends[c].data_ptr()
            rt.copy([(recv_buf.ptrs[r] + int(RO[c, r] + SO[me, c, r]) * rb, base + int(SD[me, c, r]) * rb,
                      int(R[me, c, r]) * rb) for r in range(ws)], comm)
            self._barrier(comm, dev)
            ev_sent.append(rt.record(comm))
        recv_local = rt.view(recv_buf.local, (recv_buf.bytes // rb, d), x.dtype, dev)
        ret_local = rt.view(ret_buf.local, (ret_buf.bytes // rb, d), x.dtype, dev)
        backs, ev_back = [], []
        for c in range(C):
            mark(f"wait_sent{c}_before")
            rt.wait(comp, ev_sent[c])
            mark(f"wait_sent{c}_after")
            n_recv = int(recv_c[c, me])
            rows = recv_local[int(RO[c, me]):int(RO[c, me]) + n_recv]
            rg = self.k.ep_regroup_plan(rc_me[:, c, :].contiguous(), capacity, n_recv,
                                        pos_base=None if pos_dev is None else pos_dev[c])
            xe = self.k.permute_rows(rows, rg["row_src"], rg["offsets"], rg["rows_cap"])
            mark(f"experts{c}_start")
            y = experts(xe, rg["offsets"])
            mark(f"experts{c}_end")
            backs.append(self.k.gather_rows(y, rg["recv_dst"], n_recv))
            ev_back.append(rt.record(comp))
        self.last_rows = kept_rows(Gh[:, :, me, :].sum((0, 1)), capacity)
        ev_ret = []
        for c in range(C):
            rt.wait(comm, ev_back[c])
            rt.keep(backs[c], comm)
            base = backs[c].data_ptr()
            rt.copy([(ret_buf.ptrs[s] + int(SRO[s, c] + SD[s, c, me]) * rb, base + int(SO[s, c, me]) * rb,
                      int(R[s, c, me]) * rb) for s in range(ws)], comm)
            self._barrier(comm, dev)
            ev_ret.append(rt.record(comm))
        out = torch.empty_like(x)
        mark("combine_start")
        for c, (a, b) in enumerate(bounds):
            mark(f"wait_ret{c}_before")
            rt.wait(comp, ev_ret[c])
            mark(f"wait_ret{c}_after")
            ret = ret_local[int(SRO[me, c]):int(SRO[me, c] + send_c[me, c])]
            self.k.combine(ret, plans[c]["slot_row"], w[a:b], b - a, k,
                           shared=None if shared is None else shared[a:b], out=out[a:b])
        return out

    def _fan_out(self, groups, base, keep, dev):
        """Issue each group of copies (a list of (dst, src, bytes)) on its own stream, so
        several copy engines work at once -- one group per peer; `base` waits for all of
        them.  `keep`: the source tensor, or a list of them."""
        rt = self.rt
        groups = [[sg for sg in g if sg[2] > 0] for g in groups]
        groups = [g for g in groups if g]
        streams = rt.copy_streams(dev, len(groups))
        start = rt.record(base)
        done = []
        keep = keep if isinstance(keep, (list, tuple)) else [keep]
        for g, st in zip(groups, streams):
            rt.wait(st, start)
            for t in keep:
                rt.keep(t, st)
            rt.copy(g, st)
            done.append(rt.record(st))
        for e in done:
            rt.wait(base, e)

    def _forward_p2p_local_first(self, x, idx, w, capacity, experts, shared=None, timer=None):
        """Local-first schedule.  The rows this rank routes to its OWN experts are
        contiguous in its send buffer and need no exchange.  They are computed before the
        host waits for the count matrix, so the count exchange, the host's bookkeeping and
        the copies of every other rank's rows over NVLink (one copy stream per peer) run
        underneath them.  From ``split_min_ws`` ranks on, only the first half of each
        local expert's rows goes first and the second half is computed after the other
        ranks' rows, straight into the return buffer, while the other ranks finish their
        returns.

        The sender places its rows directly in the receiver's expert-major layout (one
        copy per destination expert: local expert, then source rank, then token order),
        so the receiver's GEMM reads its receive buffer as it is -- no regrouping pass.
        With a capacity the sender knows from the count matrix which prefix of each
        segment the receiver keeps, sends only that prefix and zeroes the return rows
        of the rest; a rank's own rows for expert e follow the rows of every lower rank
        in e's (source rank, token, slot) order, so the first half of them is computed
        speculatively and the rows past the cut are zeroed the same way.

        The outputs of the other ranks' rows go back without a separate pass: the expert
        GEMM's epilogue stores each row at its address in the source rank's return
        buffer (``return_mode="fused"``; addresses from ``ep_return_rows``), so the
        return traffic crosses NVLink tile by tile while the GEMM runs.
        ``return_mode="copy"`` computes them locally and copies them back per segment
        with the copy engines."""
        rt = self.rt
        ws, El, E, me = self.world_size, self.exp_per_rank, self.num_experts, self.rank
        T, k = idx.shape
        d = x.shape[1]
        dev = x.device
        rb = d * x.element_size()
        comp, comm = rt.compute(dev), rt.comm(dev)
        recv_buf, ret_buf = self._peer_buffers(dev)

        def mark(name):
            if timer is not None:
                timer(name)

        plan = self.k.dispatch_plan(idx, E)
        send = self.k.permute_rows(x, plan["row_token"], plan["offsets"], plan["rows_cap"])
        # count exchange and its host copy on the communication stream; the host waits
        # for these alone, not for the expert work queued on the compute stream below
        G = torch.empty((ws, E), dtype=torch.int32, device=dev)
        if self._host is None or self._host.numel() < ws * E:
            self._host = rt.host_buffer(ws * E, torch.int32)
        mark("counts_start")
        rt.join(comm, comp)
        with rt.on(comm):
            dist.all_gather_into_tensor(G.view(-1), plan["counts"], group=self.group)
            self._host[:ws * E].copy_(G.view(-1), non_blocking=True)
            ev_counts = rt.record(comm)
        mark("counts_done")
        offs = plan["offsets"][me * El:(me + 1) * El + 1]
        starts, fins = offs[:-1], offs[1:]
        split = ws >= self.split_min_ws
        mids = starts + (fins - starts) // 2 if split else fins
        mark("experts_selfA_start")
        y_a = experts(send, starts, ends=mids)
        mark("experts_selfA_end")
        ev_a = rt.record(comp)
        mark("host_wait")       # the compute stream idles from here until the host enqueues again
        rt.host_wait(ev_counts)
        Gh = self._host[:ws * E].numpy().reshape(ws, ws, El).astype(np.int64)   # [src, dst, El]
        R = Gh.sum(2)                                  # slots src -> dst
        SD = np.cumsum(R, 1) - R                       # dst segment start in src's send / return layout
        W = np.cumsum(Gh, 2) - Gh                      # expert start inside the (src -> dst) segment
        if capacity > 0:                               # kept prefix of each (src, dst, expert) segment
            Kp = np.clip(capacity - (np.cumsum(Gh, 0) - Gh), 0, Gh)
        else:
            Kp = Gh
        Kr = Kp.copy()
        Kr[np.arange(ws), np.arange(ws), :] = 0        # a rank's own rows are not copied
        per_exp = Kr.sum(0)                            # [dst, El] rows each receiver gets per expert
        EO = np.cumsum(per_exp, 1) - per_exp           # expert region start in dst's receive buffer
        SO = np.cumsum(Kr, 0) - Kr                     # src offset inside that expert region
        recv_tot = per_exp.sum(1)
        send_tot = R.sum(1)
        recv_buf.ensure(int(max(recv_tot.max(), 1)) * rb)
        ret_buf.ensure(int(max(send_tot.max(), 1)) * rb)
        # dispatch: one copy per (peer, expert) segment into the peer's expert-major
        # layout, one stream per peer, then one all-reduce to order them before use
        sbase = send.data_ptr()
        self._fan_out([[(recv_buf.ptrs[r] + int(EO[r, le] + SO[me, r, le]) * rb,
                         sbase + int(SD[me, r] + W[me, r, le]) * rb, int(Kr[me, r, le]) * rb) for le in range(El)]
                       for r in range(ws) if r != me], comm, send, dev)
        self._barrier(comm, dev)
        ev_sent = rt.record(comm)
        # own rows of the first pass: copied (communication stream, once the GEMMs are
        # done) into the return buffer, whose layout is the send layout; every slot the
        # capacity dropped -- own or sent -- becomes a zero row there
        ret_local = rt.view(ret_buf.local, (ret_buf.bytes // rb, d), x.dtype, dev)
        own, keep = Gh[me, me, :], Kp[me, me, :]
        a_e = SD[me, me] + W[me, me, :]
        h_e = own // 2 if split else own               # rows of the first pass
        rbase = ret_local.data_ptr()
        rt.wait(comm, ev_a)
        rt.keep(y_a, comm)
        rt.copy([(rbase + int(a) * rb, y_a.data_ptr() + int(a) * rb, int(min(h, kp)) * rb)
                 for a, h, kp in zip(a_e, h_e, keep)], comm)
        if capacity > 0:
            with rt.on(comm):
                for r in range(ws):
                    for le in np.nonzero(Kp[me, r] < Gh[me, r])[0]:
                        a = int(SD[me, r] + W[me, r, le])
                        ret_local[a + int(Kp[me, r, le]):a + int(Gh[me, r, le])].zero_()
        # the other ranks' rows, already grouped by local expert
        mark("wait_sent0_before")
        rt.wait(comp, ev_sent)
        mark("wait_sent0_after")
        n_recv = int(recv_tot[me])
        recv_local = rt.view(recv_buf.local, (recv_buf.bytes // rb, d), x.dtype, dev)
        xe = recv_local[:n_recv]
        # one pinned table per step: expert offsets of the receive buffer, then the return
        # segments (local expert, source) -- starts, end, addresses in the sources' buffers.
        # It is rewritten only after this step's count exchange, which follows every use
        # of it by the previous step's compute stream.
        nseg = El * ws
        n_tab = 2 * nseg + 1 + El + 1 + El
        if self._seg_host is None or self._seg_host.numel() != n_tab:
            self._seg_host = rt.host_buffer(n_tab, torch.int64)
        tab = self._seg_host.numpy()
        seg_start = (EO[me][:, None] + SO[:, me, :].T).reshape(-1)          # (le, src) order
        seg_addr = [0 if s_ == me else ret_buf.ptrs[s_] + int(SD[s_, me] + W[s_, me, le]) * rb
                    for le in range(El) for s_ in range(ws)]
        tab[:nseg] = seg_start
        tab[nseg] = n_recv
        tab[nseg + 1:2 * nseg + 1] = seg_addr
        tab[2 * nseg + 1:2 * nseg + 1 + El] = EO[me]
        tab[2 * nseg + 1 + El] = n_recv
        tab[2 * nseg + 2 + El:] = keep                                       # own rows kept
        tab_dev = torch.empty(n_tab, dtype=torch.int64, device=dev)
        tab_dev.copy_(self._seg_host, non_blocking=True)
        x_offs = tab_dev[2 * nseg + 1:2 * nseg + 2 + El].to(torch.int32)
        self.last_rows = int(Kp[:, me, :].sum())
        if self.return_mode == "fused" and rb % 16 == 0:
            # the expert GEMM's epilogue stores every output row straight into its source
            # rank's return buffer (peer memory over NVLink) while the GEMM runs
            row_ptrs = self.k.ep_return_rows(None, x_offs, None, n_recv, tab_dev[:2 * nseg + 1], rb, n_recv)
            mark("experts0_start")
            experts(xe, x_offs, row_ptrs=row_ptrs)
            mark("experts0_end")
            rt.join(comm, comp)
        else:
            mark("experts0_start")
            y = experts(xe, x_offs)
            mark("experts0_end")
            rt.join(comm, comp)
            ybase = y.data_ptr()
            self._fan_out([[(seg_addr[le * ws + s_], ybase + int(seg_start[le * ws + s_]) * rb,
                             int(Kr[s_, me, le]) * rb) for le in range(El)]
                           for s_ in range(ws) if s_ != me], comm, y, dev)
        self._barrier(comm, dev)
        ev_ret = rt.record(comm)
        if split:  # second half of the kept own rows, straight into the return buffer
            ends_b = fins
            if capacity > 0:
                kd = tab_dev[2 * nseg + 2 + El:].to(torch.int32)
                ends_b = torch.maximum(mids, torch.minimum(fins, starts + kd))
            mark("experts_selfB_start")
            experts(send, mids, ends=ends_b, out=ret_local)
            mark("experts_selfB_end")
        mark("combine_start")
        mark("wait_ret0_before")
        rt.wait(comp, ev_ret)
        mark("wait_ret0_after")
        return self.k.combine(ret_local[:int(send_tot[me])], plan["slot_row"], w, T, k, shared=shared)

    # ------------------------------------------------------------ device schedule
    def reserve(self, max_tokens: int, k: int, dev) -> None:
        """Collective: size the device schedule's peer buffers for batches of up to
        ``max_tokens`` tokens on every rank (the largest value any rank passes wins).
        Called by the first device-schedule forward with its batch size; call it up
        front when later batches may be larger."""
        t = torch.tensor([int(max_tokens)], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        self.max_tokens = max(int(t.item()), 1)
        self._dev = None
        self._reserved_k = k

    def _device_state(self, k: int, row_bytes: int, dev):
        """Peer buffers sized for ``max_tokens`` and the persistent layout tensors."""
        ws, El, E = self.world_size, self.exp_per_rank, self.num_experts
        recv_rows = ws * self.max_tokens * min(k, El)        # rows one rank can receive at most
        ret_rows = self.max_tokens * k                       # this rank's send layout
        recv_buf, ret_buf = self._peer_buffers(dev)
        recv_buf.ensure(recv_rows * row_bytes)
        ret_buf.ensure(ret_rows * row_bytes)
        key = (recv_buf.local, ret_buf.local, k, row_bytes, str(dev))
        if self._dev is None or self._dev["key"] != key:
            nseg = El * ws
            i64 = dict(dtype=torch.int64, device=dev)
            i32 = dict(dtype=torch.int32, device=dev)
            self._dev = dict(
                key=key, recv_rows=recv_rows, ret_rows=ret_rows,
                recv_base=torch.tensor(recv_buf.ptrs, **i64), ret_base=torch.tensor(ret_buf.ptrs, **i64),
                G=torch.zeros((ws, E), **i32),
                lay=dict(send_addr=torch.zeros(E, **i64), keep=torch.zeros(E, **i32),
                         recv_offsets=torch.zeros(El + 1, **i32), seg=torch.zeros(2 * nseg + 1, **i64)),
                send=None)
        return self._dev, recv_buf, ret_buf

    def _forward_p2p_device(self, x, idx, w, capacity, experts, shared=None, timer=None):
        """Device schedule: the host never waits for the device.

        * compute stream: plan (rows grouped by global expert); this rank's own rows
          permuted into the send buffer and run through its experts straight into the
          return buffer (their rows there follow the send layout);
        * communication stream, meanwhile: the per-expert counts of every rank
          all-gathered into device memory, ``ep_layout`` turning them into addresses
          (each segment's place in its owner's expert-major receive buffer, the kept
          prefix under the capacity cut, this rank's receive offsets and the return
          address of every received segment), ``ep_send_rows`` storing every routed row
          of the other ranks' experts from x straight into the owners' receive buffers
          over NVLink, then a one-int all-reduce that orders those stores before every
          rank's next step;
        * compute stream: the experts over the received rows (offsets read from device
          memory), whose epilogue stores each output row into its source rank's return
          buffer (fused return); an all-reduce, then the combine over the return buffer
          (slots the capacity cut dropped are marked -1 first).

        Buffers are sized for ``max_tokens`` tokens per rank (set by the first forward
        or by ``reserve``), so no size depends on this batch's routing."""
        rt = self.rt
        ws, El, E, me = self.world_size, self.exp_per_rank, self.num_experts, self.rank
        T, k = idx.shape
        d = x.shape[1]
        dev = x.device
        rb = d * x.element_size()
        if rb % 16:
            raise ValueError("the device schedule needs rows of a multiple of 16 bytes")
        if self.max_tokens is None or getattr(self, "_reserved_k", k) != k:
            self.reserve(T, k, dev)
        if T > self.max_tokens:
            from ._lib import SwiftMoEError
            raise SwiftMoEError(f"batch of {T} tokens exceeds the exchange's max_tokens={self.max_tokens}; "
                                f"call reserve() with the largest batch on every rank first")
        comp, comm = rt.compute(dev), rt.comm(dev)

        def mark(name):
            if timer is not None:
                timer(name)

        st, recv_buf, ret_buf = self._device_state(k, rb, dev)
        lay, G = st["lay"], st["G"]
        plan = self.k.dispatch_plan(idx, E)
        rows_cap = plan["rows_cap"]
        send = st["send"]
        if send is None or send.shape[0] < rows_cap or send.dtype != x.dtype:
            send = st["send"] = torch.empty((max(self.max_tokens * k, 1), d), dtype=x.dtype, device=dev)
        own = plan["offsets"][me * El:(me + 1) * El + 1]
        self.k.permute_rows(x, plan["row_token"], own, rows_cap, out=send)
        mark("counts_start")
        rt.join(comm, comp)
        for t in (x, plan["row_token"], plan["offsets"], plan["counts"]):
            rt.keep(t, comm)
        with rt.on(comm):
            dist.all_gather_into_tensor(G.view(-1), plan["counts"], group=self.group)
            self.k.ep_layout(G, me, capacity, st["recv_base"], st["ret_base"], rb, st["recv_rows"], lay)
            self.k.ep_send_rows(x, plan["row_token"], plan["offsets"], me * El, El, lay["send_addr"], lay["keep"],
                                rows_cap)
        self._barrier(comm, dev)
        ev_sent = rt.record(comm)
        mark("counts_done")
        ret_local = rt.view(ret_buf.local, (st["ret_rows"], d), x.dtype, dev)
        mark("experts_self_start")
        experts(send, own[:-1], ends=own[1:], out=ret_local)
        mark("experts_self_end")
        mark("wait_sent0_before")
        rt.wait(comp, ev_sent)
        mark("wait_sent0_after")
        if capacity > 0:
            self.k.ep_drop_slots(idx, plan["offsets"], lay["keep"], plan["slot_row"])
        recv_local = rt.view(recv_buf.local, (st["recv_rows"], d), x.dtype, dev)
        R = st["recv_rows"]
        row_ptrs = self.k.ep_return_rows(None, lay["recv_offsets"], None, R, lay["seg"], rb, R)
        mark("experts0_start")
        experts(recv_local, lay["recv_offsets"], row_ptrs=row_ptrs)
        mark("experts0_end")
        self._rows_dev = (lay["keep"][me * El:(me + 1) * El].sum().view(1), lay["recv_offsets"][El:])
        rt.join(comm, comp)
        self._barrier(comm, dev)
        ev_ret = rt.record(comm)
        mark("combine_start")
        mark("wait_ret0_before")
        rt.wait(comp, ev_ret)
        mark("wait_ret0_after")
        return self.k.combine(ret_local[:max(T * k, 1)], plan["slot_row"], w, T, k, shared=shared)

    def _forward_p2p_device_dedup(self, x, idx, w, experts, shared=None, timer=None):
        """Token dedup on the device schedule: no host wait.  The rows and their slot
        metadata are those of ``_forward_p2p_dedup`` (one row per (token, rank), this
        rank's rotated rank order with its own rank first, each sent row carrying the
        local expert and gate weight of the token's k slots); their layout in the
        receivers' buffers comes from ``ep_layout`` in its rotated mode (rows, then
        expert ids, then weights, one call each), the send kernel stores all three into
        the peers, the receiver marks its unfilled rows, expands, runs the experts and
        stores one weighted partial row per received row straight back into its
        source's return buffer; the own rows' partial sums are copied into the own
        segment.  Buffers are sized for ``max_tokens`` tokens per rank."""
        rt = self.rt
        ws, El, E, me = self.world_size, self.exp_per_rank, self.num_experts, self.rank
        T, k = idx.shape
        d = x.shape[1]
        dev = x.device
        rb = d * x.element_size()
        if self.max_tokens is None or getattr(self, "_reserved_k", k) != k:
            self.reserve(T, k, dev)
        if T > self.max_tokens:
            from ._lib import SwiftMoEError
            raise SwiftMoEError(f"batch of {T} tokens exceeds the exchange's max_tokens={self.max_tokens}; "
                                f"call reserve() with the largest batch on every rank first")
        comp, comm = rt.compute(dev), rt.comm(dev)

        def mark(name):
            if timer is not None:
                timer(name)

        st, recv_buf, ret_buf = self._dedup_state(k, rb, dev)
        R = st["recv_rows"]
        ridx = self.k.ep_dedup_ranks(idx, El, ws, me)
        rplan = self.k.dispatch_plan(ridx, ws)                    # one row per (token, rank), own rank first
        rows_cap = rplan["rows_cap"]
        meta_e, meta_w, own_e = self.k.ep_dedup_meta(idx, w, ridx, rplan["slot_row"], rplan["counts"][0:1], El, ws,
                                                     rows_cap)
        ident = st["ident"][:max(rows_cap, 1)]
        G = st["G"]
        mark("counts_start")
        rt.join(comm, comp)
        for t in (x, rplan["row_token"], rplan["offsets"], rplan["counts"], meta_e, meta_w):
            rt.keep(t, comm)
        with rt.on(comm):
            dist.all_gather_into_tensor(G.view(-1), rplan["counts"], group=self.group)
            for lay, base, nb in ((st["lay_x"], st["recv_base"], rb), (st["lay_e"], st["recv_base_e"], 4 * k),
                                  (st["lay_w"], st["recv_base_w"], 4 * k)):
                self.k.ep_layout(G, me, 0, base, st["ret_base"], nb, R, lay, rotated=True)
            self.k.ep_send_rows(x, rplan["row_token"], rplan["offsets"], 0, 1, st["lay_x"]["send_addr"],
                                st["lay_x"]["keep"], rows_cap)
            self.k.ep_send_rows(meta_e, ident, rplan["offsets"], 0, 1, st["lay_e"]["send_addr"], st["lay_e"]["keep"],
                                rows_cap)
            self.k.ep_send_rows(meta_w, ident, rplan["offsets"], 0, 1, st["lay_w"]["send_addr"], st["lay_w"]["keep"],
                                rows_cap)
        self._barrier(comm, dev)
        ev_sent = rt.record(comm)
        mark("counts_done")
        # own rows: expand, compute, weighted partial sums into the own segment of the
        # return buffer (rows [0, own count) of the send layout)
        send = self.k.permute_rows(x, rplan["row_token"], rplan["offsets"][0:2], rows_cap)
        oplan = self.k.dispatch_plan(own_e[:T], El)
        xo = self.k.permute_rows(send, oplan["row_token"], oplan["offsets"], oplan["rows_cap"])
        mark("experts_self_start")
        yo = experts(xo, oplan["offsets"])
        mark("experts_self_end")
        part_own = self.k.combine(yo, oplan["slot_row"], meta_w[:T], T, k)
        ret_local = rt.view(ret_buf.local, (st["ret_rows"], d), x.dtype, dev)
        self.k.copy_rows_count(ret_local, part_own, rplan["counts"][0:1])
        mark("wait_sent0_before")
        rt.wait(comp, ev_sent)
        mark("wait_sent0_after")
        n_recv = st["lay_x"]["recv_offsets"][1:2]
        xr = rt.view(recv_buf.local, (R, d), x.dtype, dev)
        er = rt.view(recv_buf.local + st["off_e"], (R, k), torch.int32, dev)
        wr = rt.view(recv_buf.local + st["off_w"], (R, k), torch.float32, dev)
        self.k.ep_clear_tail(er, n_recv)
        rp = self.k.dispatch_plan(er, El)
        xe = self.k.permute_rows(xr, rp["row_token"], rp["offsets"], rp["rows_cap"])
        mark("experts0_start")
        y = experts(xe, rp["offsets"])
        mark("experts0_end")
        part = self.k.combine(y, rp["slot_row"], wr, R, k)
        row_ptrs = self.k.ep_return_rows(None, st["lay_x"]["recv_offsets"], None, R, st["lay_x"]["seg"], rb, R)
        self.k.store_rows(part, row_ptrs, R)
        self._rows_dev = (oplan["offsets"][El:], rp["offsets"][El:])
        rt.join(comm, comp)
        self._barrier(comm, dev)
        ev_ret = rt.record(comm)
        mark("combine_start")
        mark("wait_ret0_before")
        rt.wait(comp, ev_ret)
        mark("wait_ret0_after")
        if self._ones is None or self._ones.shape != (T, k) or self._ones.device != dev:
            self._ones = torch.ones((T, k), dtype=torch.float32, device=dev)
        return self.k.combine(ret_local[:max(rows_cap, 1)], rplan["slot_row"], self._ones, T, k, shared=shared)

    def _dedup_state(self, k: int, row_bytes: int, dev):
        """Peer buffers of the dedup device schedule (rows, then per-slot expert ids, then
        weights, in one receive buffer) and its persistent layout tensors."""
        ws = self.world_size
        R = max((ws - 1) * self.max_tokens, 1)               # rows one rank can receive at most
        ret_rows = self.max_tokens * min(k, ws)               # (token, rank) rows of the send layout
        al = lambda v: (v + 255) // 256 * 256
        off_e = al(R * row_bytes)
        off_w = off_e + al(R * k * 4)
        recv_buf, ret_buf = self._peer_buffers(dev)
        recv_buf.ensure(off_w + R * k * 4)
        ret_buf.ensure(ret_rows * row_bytes)
        key = ("dedup", recv_buf.local, ret_buf.local, k, row_bytes, str(dev))
        if self._dev is None or self._dev.get("key") != key:
            i64 = dict(dtype=torch.int64, device=dev)
            i32 = dict(dtype=torch.int32, device=dev)
            lay = lambda: dict(send_addr=torch.zeros(ws, **i64), keep=torch.zeros(ws, **i32),
                               recv_offsets=torch.zeros(2, **i32), seg=torch.zeros(2 * ws + 1, **i64))
            self._dev = dict(
                key=key, recv_rows=R, ret_rows=ret_rows, off_e=off_e, off_w=off_w,
                recv_base=torch.tensor(recv_buf.ptrs, **i64), ret_base=torch.tensor(ret_buf.ptrs, **i64),
                recv_base_e=torch.tensor([p_ + off_e for p_ in recv_buf.ptrs], **i64),
                recv_base_w=torch.tensor([p_ + off_w for p_ in recv_buf.ptrs], **i64),
                G=torch.zeros((ws, ws), **i32), lay_x=lay(), lay_e=lay(), lay_w=lay(),
                ident=torch.arange(max(self.max_tokens * min(k, ws), 1), **i32))
        return self._dev, recv_buf, ret_buf

    def _forward_p2p_dedup(self, x, idx, w, experts, shared=None, timer=None):
        """Local-first schedule with token dedup, for top-k routing with several experts
        per rank (no capacity).  Each token travels once to each rank that owns any of
        its experts, with the local expert and gate weight of each of its k slots (-1 /
        0 for slots bound elsewhere): ``ep_dedup_ranks`` + a dispatch plan over ranks lay
        out one send row per (token, rank), this rank's own rows first.  The receiver
        expands the rows into expert-major slot rows (dispatch plan over the received
        local experts + permute), runs the experts and returns ONE gate-weighted partial
        sum per received row (combine); the sender adds the partial sums of its token's
        ranks (combine with unit weights over the rank plan).  The own rows go through
        the same expansion on the compute stream before the host waits for the count
        matrix, underneath the count exchange and the dispatch copies.

        With k slots spread over the ranks a token crosses NVLink once per distinct rank
        instead of once per slot (with 128 experts and k = 8: about 2 rows instead of 8
        at 2 ranks, 5.3 instead of 7 remote slots at 8), in exchange for a permute on the
        receiver and partial sums rounded to the compute dtype."""
        rt = self.rt
        ws, El, E, me = self.world_size, self.exp_per_rank, self.num_experts, self.rank
        T, k = idx.shape
        d = x.shape[1]
        dev = x.device
        rb = d * x.element_size()
        comp, comm = rt.compute(dev), rt.comm(dev)
        recv_buf, ret_buf = self._peer_buffers(dev)

        def mark(name):
            if timer is not None:
                timer(name)

        ridx = self.k.ep_dedup_ranks(idx, El, ws, me)
        rplan = self.k.dispatch_plan(ridx, ws)                    # one row per (token, rank)
        send = self.k.permute_rows(x, rplan["row_token"], rplan["offsets"], rplan["rows_cap"])
        meta_e, meta_w, own_e = self.k.ep_dedup_meta(idx, w, ridx, rplan["slot_row"], rplan["counts"][0:1], El, ws,
                                                     rplan["rows_cap"])
        G = torch.empty((ws, ws), dtype=torch.int32, device=dev)   # [src, rotated destination]
        if self._host is None or self._host.numel() < ws * ws:
            self._host = rt.host_buffer(ws * ws, torch.int32)
        mark("counts_start")
        rt.join(comm, comp)
        with rt.on(comm):
            dist.all_gather_into_tensor(G.view(-1), rplan["counts"], group=self.group)
            self._host[:ws * ws].copy_(G.view(-1), non_blocking=True)
            ev_counts = rt.record(comm)
        mark("counts_done")
        # own rows: expand, compute, weighted partial sums (compute stream, no host wait)
        oplan = self.k.dispatch_plan(own_e[:T], El)
        xo = self.k.permute_rows(send, oplan["row_token"], oplan["offsets"], oplan["rows_cap"])
        mark("experts_selfA_start")
        yo = experts(xo, oplan["offsets"])
        mark("experts_selfA_end")
        part_own = self.k.combine(yo, oplan["slot_row"], meta_w[:T], T, k)
        ev_a = rt.record(comp)
        mark("host_wait")
        rt.host_wait(ev_counts)
        Gc = self._host[:ws * ws].numpy().reshape(ws, ws).astype(np.int64)
        ex = np.cumsum(Gc, 1) - Gc
        R = np.stack([np.roll(Gc[s_], s_) for s_ in range(ws)])       # [src, dst] rows
        SDr = np.stack([np.roll(ex[s_], s_) for s_ in range(ws)])     # dst segment start in src's layout
        Rr = R.copy()
        np.fill_diagonal(Rr, 0)
        SO = np.cumsum(Rr, 0) - Rr                     # src offset in dst's receive layout
        recv_tot, send_tot = Rr.sum(0), R.sum(1)
        n_max = int(max(recv_tot.max(), 1))
        al = lambda v: (v + 255) // 256 * 256
        off_e = al(n_max * rb)                         # receive buffer: rows, local experts, weights
        off_w = off_e + al(n_max * k * 4)
        recv_buf.ensure(off_w + n_max * k * 4)
        ret_buf.ensure(int(max(send_tot.max(), 1)) * rb)
        sb, eb, wb = send.data_ptr(), meta_e.data_ptr(), meta_w.data_ptr()
        groups = []
        for r in range(ws):
            if r == me:
                continue
            n, so, sd = int(R[me, r]), int(SO[me, r]), int(SDr[me, r])
            groups.append([(recv_buf.ptrs[r] + so * rb, sb + sd * rb, n * rb),
                           (recv_buf.ptrs[r] + off_e + so * k * 4, eb + sd * k * 4, n * k * 4),
                           (recv_buf.ptrs[r] + off_w + so * k * 4, wb + sd * k * 4, n * k * 4)])
        self._fan_out(groups, comm, [send, meta_e, meta_w], dev)
        self._barrier(comm, dev)
        ev_sent = rt.record(comm)
        ret_local = rt.view(ret_buf.local, (ret_buf.bytes // rb, d), x.dtype, dev)
        rt.wait(comm, ev_a)                            # own partial sums: the first segment
        rt.keep(part_own, comm)
        rt.copy([(ret_local.data_ptr(), part_own.data_ptr(), int(R[me, me]) * rb)], comm)
        # the other ranks' rows
        mark("wait_sent0_before")
        rt.wait(comp, ev_sent)
        mark("wait_sent0_after")
        n_recv = int(recv_tot[me])
        xr = rt.view(recv_buf.local, (n_max, d), x.dtype, dev)[:n_recv]
        er = rt.view(recv_buf.local + off_e, (n_max, k), torch.int32, dev)[:n_recv]
        wr = rt.view(recv_buf.local + off_w, (n_max, k), torch.float32, dev)[:n_recv]
        rp = self.k.dispatch_plan(er, El)
        xe = self.k.permute_rows(xr, rp["row_token"], rp["offsets"], rp["rows_cap"])
        mark("experts0_start")
        y = experts(xe, rp["offsets"])
        mark("experts0_end")
        part = self.k.combine(y, rp["slot_row"], wr, n_recv, k)
        self._rows_dev = (oplan["offsets"][El:], rp["offsets"][El:])
        rt.join(comm, comp)
        pb = part.data_ptr()
        self._fan_out([[(ret_buf.ptrs[s_] + int(SDr[s_, me]) * rb, pb + int(SO[s_, me]) * rb, int(R[s_, me]) * rb)]
                       for s_ in range(ws) if s_ != me], comm, [part], dev)
        self._barrier(comm, dev)
        ev_ret = rt.record(comm)
        mark("combine_start")
        mark("wait_ret0_before")
        rt.wait(comp, ev_ret)
        mark("wait_ret0_after")
        if self._ones is None or self._ones.shape != (T, k) or self._ones.device != dev:
            self._ones = torch.ones((T, k), dtype=torch.float32, device=dev)
        return self.k.combine(ret_local[:int(send_tot[me])], rplan["slot_row"], self._ones, T, k, shared=shared)

    def close(self):
        """Collective: release the peer buffers of the p2p transport."""
        if self._bufs is not None:
            for b in self._bufs:
                b.release()
            self._bufs = None

    # ------------------------------------------------------------------ stage API
    def dispatch(self, x: torch.Tensor, idx: torch.Tensor, capacity: int = 0,
                 slot_payload: Optional[torch.Tensor] = None):
        """Unchunked dispatch for the stage-by-stage API (StandardMoE._dispatch_tokens):
        returns (rows grouped by local expert, expert offsets [E_l+1], state).

        ``slot_payload`` (optional, float32 [T, k]: one value per (token, slot), e.g. the
        gate weights): travels with the rows, as the reference sends its weights next to
        its rows (models/baseline_moe.py:131-133); returned as a fourth value, one entry
        per returned row."""
        ws, El = self.world_size, self.exp_per_rank
        T, k = idx.shape
        plan = self.k.dispatch_plan(idx, self.num_experts)
        send_rows = self.k.permute_rows(x, plan["row_token"], plan["offsets"], plan["rows_cap"])
        counts = plan["counts"]
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts)
        hc, hr = self._to_host(counts, recv_counts)
        send_splits = [int(v) for v in hc.reshape(ws, El).sum(1)]
        recv_splits = [int(v) for v in hr.reshape(ws, El).sum(1)]
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        recv_rows = torch.empty((max(n_recv, 1), x.shape[1]), dtype=x.dtype, device=x.device)
        self._a2a(recv_rows[:n_recv], send_rows[:n_send], recv_splits, send_splits)
        rg = self.k.ep_regroup_plan(recv_counts.view(ws, El), capacity, n_recv)
        xe = self.k.permute_rows(recv_rows, rg["row_src"], rg["offsets"], rg["rows_cap"])
        st = DispatchState(plan, rg, send_splits, recv_splits, n_send, n_recv, T, k)
        if slot_payload is None:
            return xe, rg["offsets"], st
        # payload of every send row: the value of the (token, slot) that row holds
        flat = slot_payload.reshape(-1).float()
        sr = plan["slot_row"].reshape(-1).long()
        send_p = torch.zeros(n_send + 1, dtype=torch.float32, device=x.device)   # last: spare for skipped slots
        send_p.scatter_(0, torch.where(sr >= 0, sr, torch.full_like(sr, n_send)), flat)
        recv_p = torch.empty(max(n_recv, 1), dtype=torch.float32, device=x.device)
        self._a2a(recv_p[:n_recv], send_p[:n_send], recv_splits, send_splits)
        pe = self.k.gather_rows(recv_p.view(-1, 1), rg["row_src"], rg["rows_cap"])
        return xe, rg["offsets"], st, pe.view(-1)

    def return_rows(self, y: torch.Tensor, st: DispatchState) -> torch.Tensor:
        """Rows computed for the rows ``dispatch`` delivered (``y`` in its expert-major order,
        any width and dtype) back to their source ranks: [n_send, width] in each source's
        send layout (row ``st.plan["slot_row"][t*k + j]`` for slot j of token t), zero rows
        for the slots the capacity cut dropped."""
        back = self.k.gather_rows(y, st.regroup["recv_dst"], st.n_recv)
        ret = torch.empty((max(st.n_send, 1), y.shape[1]), dtype=y.dtype, device=y.device)
        self._a2a(ret[:st.n_send], back[:st.n_recv], st.send_splits, st.recv_splits)
        return ret

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None) -> None:
        """all_to_all_single over the group; a local copy on a one-rank group."""
        if self.world_size == 1:
            if out.numel():
                out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def combine(self, y: torch.Tensor, st: DispatchState, w: torch.Tensor,
                shared: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
        """Return expert outputs to their source ranks and reduce the k slots."""
        ret = self.return_rows(y, st)
        return self.k.combine(ret, st.plan["slot_row"], w, st.T, st.k, shared=shared, out=out)

    def layer_backward(self, x: torch.Tensor, dout: torch.Tensor, gate: torch.Tensor,
                       logit_bias: Optional[torch.Tensor], k: int, capacity: int, experts: dict,
                       shared: Optional[dict] = None) -> dict:
        """Gradients of the expert-parallel layer for the upstream gradient ``dout`` of this
        rank's tokens ``x`` [T, d] (16-bit on the GPU).

        The routed rows' part runs where their experts live, the tokens' part here, as the
        one-GPU ``smoe_layer_bwd`` splits it: the routing is recomputed, the rows of x and
        of dout travel to the experts' ranks (the forward's dispatch, capacity cut
        included, with the gate weights beside the dout rows), the owner recomputes the
        gate/up pre-activations, runs the SwiGLU (or linear) backward, the input-gradient
        GEMM and the weight-gradient GEMMs over its local experts (rows padded to 64 per
        expert for the K-grouped GEMM), and returns one input-gradient row and one gate-
        weight gradient per slot; this rank then adds the slots, the router's softmax-over-
        top-k backward and the shared expert.

        ``experts``: ``{"kind": "swiglu", "w1", "w3" [E_l, F, d], "w2t" [E_l, F, d] (W2
        transposed), "w13t" [E_l, d, 2F] ([W1; W3] transposed)}`` or ``{"kind": "linear",
        "w": [E_l, d, d] (the B operand of the dout GEMM), "transposed": bool (weights used
        as x @ W)}``; ``shared`` (optional): ``{"w1", "w3" [1, Fs, d], "w2t" [1, Fs, d],
        "w13t" [1, d, 2Fs]}``.  Returns ``x``, ``gate`` [E, d] fp32, ``w13`` [E_l, 2F, d]
        and ``w2`` [E_l, d, F] (or ``lin`` [E_l, d, d]) fp32, ``s13`` / ``s2`` for the shared
        expert.  The gate's and the shared expert's gradients are this rank's contribution
        (those weights are replicated: sum them over ranks, as data parallelism does); the
        local experts' gradients are complete.  The routed dispatch is host-synchronised
        (the counts become Python ints), as in the stage-by-stage API."""
        kk = self.k
        El, E = self.exp_per_rank, self.num_experts
        T, d = x.shape
        dev = x.device
        f32 = dict(dtype=torch.float32, device=dev)
        idx, w = kk.router(x, gate, k, logit_bias)
        # ---- the routed rows on their experts' rank
        xe, oe, st = self.dispatch(x, idx, capacity)
        de, _, _, we = self.dispatch(dout, idx, capacity, slot_payload=w)
        n = int(oe[El])
        r = torch.arange(max(n, 1), device=dev, dtype=torch.int32)[:n]
        ids = torch.searchsorted(oe[1:].contiguous(), r, right=True).to(torch.int32)
        pa = kk.dispatch_plan(ids.view(-1, 1).contiguous(), El, 0, 64)   # groups start on 64-row boundaries
        S, offs = pa["rows_cap"], pa["offsets"]
        xa = kk.permute_rows(xe, pa["row_token"], offs, S)              # padding rows are zeros
        da = kk.permute_rows(de, pa["row_token"], offs, S)
        used = int(offs[El])                      # rows of the padded layout (padding included)
        rw = torch.zeros(max(S, 1), **f32)        # gate weight of each padded row (0 for padding)
        if used:
            rt = pa["row_token"][:used].long()    # in [0, n), or -1 for padding
            rw[:used] = torch.where(rt >= 0, we.reshape(-1)[:n].float()[rt.clamp(min=0)], torch.zeros((), **f32))
        dwr = torch.zeros(max(S, 1), **f32)
        out = {}
        if experts["kind"] == "swiglu":
            F = experts["w1"].shape[1]
            ab = torch.empty((max(S, 1), 2 * F), dtype=x.dtype, device=dev)
            kk.grouped_gemm(xa, experts["w1"], offs, B3=experts["w3"], epilogue=L.SMOE_EPI_GATEUP, out=ab)
            g = kk.grouped_gemm(da, experts["w2t"], offs)                   # dout_r W2
            kk.swiglu_bwd(ab, g, rw, offs[El:], dwr)                        # [da | db], w h, <g, h>
            dxa = kk.grouped_gemm(ab, experts["w13t"], offs)                # input gradient of the rows
            out["w13"] = kk.wgrad_gemm_rows(ab, xa, offs, 2 * F, d)
            out["w2"] = kk.wgrad_gemm_rows(da, g, offs, d, F)
        else:
            g = kk.grouped_gemm(da, experts["w"], offs)                     # dout_r Wl
            kk.linear_bwd(g, xa, da, rw, offs[El:], dwr)                    # w g, w dout, <g, x>
            dxa = g
            out["lin"] = (kk.wgrad_gemm_rows(xa, da, offs, d, d) if experts["transposed"]
                          else kk.wgrad_gemm_rows(da, xa, offs, d, d))
        # back in dispatch's row order, then to the source ranks (zero rows for dropped slots)
        sr = pa["slot_row"][:n]
        dxe = kk.gather_rows(dxa, sr, n)
        dwe = dwr[sr.long()].reshape(-1, 1).contiguous() if n else torch.zeros((1, 1), **f32)
        ret_dx = self.return_rows(dxe, st)
        ret_dw = self.return_rows(dwe, st).reshape(-1).contiguous()
        # ---- the tokens' part, here
        dxs = None
        if shared is not None:
            Fs = shared["w1"].shape[1]
            soff = torch.tensor([0, T], dtype=torch.int32, device=dev)
            abs_ = torch.empty((max(T, 1), 2 * Fs), dtype=x.dtype, device=dev)
            kk.grouped_gemm(x, shared["w1"], soff, B3=shared["w3"], epilogue=L.SMOE_EPI_GATEUP, out=abs_)
            gs = kk.grouped_gemm(dout, shared["w2t"], soff)
            kk.swiglu_bwd(abs_, gs, None, None, None)
            dxs = kk.grouped_gemm(abs_, shared["w13t"], soff)
            out["s13"] = kk.wgrad_gemm_rows(abs_, x, soff, 2 * Fs, d)[0]
            out["s2"] = kk.wgrad_gemm_rows(dout, gs, soff, d, Fs)[0]
        pf = kk.dispatch_plan(idx, E, 0)                                  # every slot, for the gate gradient
        dsel = torch.zeros(max(pf["rows_cap"], 1), **f32)
        dx = torch.empty_like(x)
        kk.moe_bwd_dx(ret_dx, st.plan["slot_row"], idx, w, ret_dw, gate, dxs, dx, pf["slot_row"], dsel)
        out["gate"] = kk.router_dwg(x, pf["row_token"], pf["offsets"], dsel, E)
        out["x"] = dx
        return out


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _maybe_stream(s):
    return torch.cuda.stream(s) if s is not None else _NullCtx()


def _record(s):
    if s is None:
        return None
    e = torch.cuda.Event()
    e.record(s)
    return e


def _wait(s, ev):
    if s is not None and ev is not None:
        s.wait_event(ev)
