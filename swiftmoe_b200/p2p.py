"""Peer buffers for the expert-parallel exchange: one device buffer per rank, allocated by
libswiftmoe, exported as a CUDA IPC handle and opened by every other rank of the node,
so that rows move with device-to-device copies over NVLink (copy engines; the SMs stay
with the expert GEMMs)."""
from __future__ import annotations

import ctypes as C
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _lib as L

HANDLE = 64
_TORCH_TO_TYPESTR = {torch.bfloat16: "<i2", torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4",
                     torch.uint8: "|u1"}


class _CudaArray:
    """Minimal __cuda_array_interface__ exporter so torch can view library memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def view(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A torch tensor over existing device memory (no copy, no ownership)."""
    t = torch.as_tensor(_CudaArray(ptr, shape, _TORCH_TO_TYPESTR[dtype]), device=device)
    return t.view(dtype) if dtype == torch.bfloat16 else t


class PeerBuffers:
    """A symmetric set of device buffers, one per rank, every one addressable by all."""

    def __init__(self, group: Optional[dist.ProcessGroup], rank: int, world_size: int, device: torch.device):
        self.group, self.rank, self.ws, self.device = group, rank, world_size, device
        self.bytes = 0
        self.local: Optional[int] = None
        self.ptrs: List[Optional[int]] = [None] * world_size

    def ensure(self, nbytes: int) -> None:
        """Collective: every rank calls it with the same size; reallocates only when the
        buffers are too small (with headroom), then re-exchanges the handles."""
        if nbytes <= self.bytes:
            return
        new = max(int(nbytes * 1.25), 1 << 21)
        new = (new + (1 << 21) - 1) // (1 << 21) << 21
        self.release()
        lib = L.load()
        p = C.c_void_p()
        h = (C.c_ubyte * HANDLE)()
        L.check(lib.smoe_ep_buffer_create(new, C.byref(p), C.cast(h, C.c_void_p)), "smoe_ep_buffer_create")
        self.local = p.value
        mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=self.device)
        allh = torch.empty(self.ws * HANDLE, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, mine, group=self.group)
        allh = allh.cpu().numpy().reshape(self.ws, HANDLE)
        for r in range(self.ws):
            if r == self.rank:
                self.ptrs[r] = self.local
                continue
            hb = (C.c_ubyte * HANDLE).from_buffer_copy(allh[r].tobytes())
            q = C.c_void_p()
            L.check(lib.smoe_ep_peer_open(C.cast(hb, C.c_void_p), C.byref(q)), "smoe_ep_peer_open")
            self.ptrs[r] = q.value
        self.bytes = new

    def release(self) -> None:
        """Collective: waits for all work and all ranks before unmapping and freeing."""
        if self.local is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group, device_ids=[self.device.index])
        lib = L.load()
        for r, q in enumerate(self.ptrs):
            if r != self.rank and q is not None:
                lib.smoe_ep_peer_close(q)
        lib.smoe_ep_buffer_destroy(self.local)
        self.local, self.ptrs, self.bytes = None, [None] * self.ws, 0


def copy_segments(segs, stream: torch.cuda.Stream) -> None:
    """segs: list of (dst_ptr, src_ptr, nbytes); one device-to-device copy each."""
    segs = [s for s in segs if s[2] > 0]
    if not segs:
        return
    n = len(segs)
    dst = (C.c_void_p * n)(*[s[0] for s in segs])
    src = (C.c_void_p * n)(*[s[1] for s in segs])
    nb = (C.c_size_t * n)(*[s[2] for s in segs])
    L.check(L.load().smoe_copy_segments(dst, src, nb, n, stream.cuda_stream), "smoe_copy_segments")


class CudaRuntime:
    """Streams, events, peer buffers and copies of the peer-copy transport on CUDA
    devices.  The exchange schedules in ep.py only talk to the device through this
    object, so a host implementation of the same methods can run them on CPU ranks."""

    def __init__(self):
        self._comm = {}
        self._copy = {}

    @staticmethod
    def compute(dev):
        return torch.cuda.current_stream(dev)

    def comm(self, dev):
        s = self._comm.get(dev.index)
        if s is None:
            s = self._comm[dev.index] = torch.cuda.Stream(dev)
        return s

    def copy_streams(self, dev, n: int):
        lst = self._copy.get(dev.index)
        if lst is None or len(lst) < n:
            lst = self._copy[dev.index] = [torch.cuda.Stream(dev) for _ in range(max(n, 1))]
        return lst[:n]

    @staticmethod
    def on(s):
        return torch.cuda.stream(s)

    @staticmethod
    def record(s):
        e = torch.cuda.Event()
        e.record(s)
        return e

    @staticmethod
    def wait(s, ev):
        s.wait_event(ev)

    @staticmethod
    def join(s, other):
        s.wait_stream(other)

    @staticmethod
    def host_wait(ev):
        ev.synchronize()

    @staticmethod
    def keep(t: torch.Tensor, s):
        t.record_stream(s)

    @staticmethod
    def host_buffer(n: int, dtype: torch.dtype) -> torch.Tensor:
        return torch.empty(n, dtype=dtype, pin_memory=True)

    @staticmethod
    def buffers(group, rank: int, world_size: int, dev: torch.device) -> PeerBuffers:
        return PeerBuffers(group, rank, world_size, dev)

    @staticmethod
    def view(ptr: int, shape, dtype: torch.dtype, dev: torch.device) -> torch.Tensor:
        return view(ptr, shape, dtype, dev)

    @staticmethod
    def copy(segs, s) -> None:
        copy_segments(segs, s)
