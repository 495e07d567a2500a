"""CPU test double of swiftmoe_b200.p2p.CudaRuntime: the peer buffers are POSIX shared
memory segments mapped by every rank process, a copy is a memmove between mapped
addresses, and streams and events are synchronous (None).  With it the peer-copy
schedules of ExpertParallelExchange run on gloo ranks without a GPU, with the same
offsets, buffer layouts and copy segments as on CUDA devices."""
import ctypes
from multiprocessing import resource_tracker, shared_memory

import numpy as np
import torch
import torch.distributed as dist


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _attach(name):
    m = shared_memory.SharedMemory(name=name)
    resource_tracker.unregister(m._name, "shared_memory")   # the creating rank owns it
    return m


class ShmBuffers:
    """Same contract as p2p.PeerBuffers: ensure() and release() are collective."""

    def __init__(self, group, rank, world_size, tag, registry):
        self.group, self.rank, self.ws, self.tag = group, rank, world_size, tag
        self.registry = registry          # local address -> shared memory (for views)
        self.bytes, self.local, self.ptrs = 0, None, [None] * world_size
        self._maps, self._pins, self.gen = [], [], 0

    def ensure(self, nbytes: int) -> None:
        if nbytes <= self.bytes:
            return
        new = max(int(nbytes * 1.25), 4096)
        self.release()
        self.gen += 1
        mine = shared_memory.SharedMemory(name=self._name(self.rank), create=True, size=new)
        dist.barrier(group=self.group)
        self._maps = [mine if r == self.rank else _attach(self._name(r)) for r in range(self.ws)]
        self._pins = [np.frombuffer(m.buf, dtype=np.uint8) for m in self._maps]
        self.ptrs = [int(a.ctypes.data) for a in self._pins]
        self.local = self.ptrs[self.rank]
        self.registry[self.local] = mine
        self.bytes = new
        dist.barrier(group=self.group)

    def _name(self, r):
        return f"{self.tag}_{self.gen}_{r}"

    def release(self) -> None:
        if self.local is None:
            return
        dist.barrier(group=self.group)
        self.registry.pop(self.local, None)
        self._pins = []
        for m in self._maps:
            try:
                m.close()
            except BufferError:      # a tensor view is still alive; unmapped at exit
                pass
        dist.barrier(group=self.group)   # every rank unmapped before the owner unlinks
        self._maps[self.rank].unlink()
        self._maps, self.local, self.ptrs, self.bytes = [], None, [None] * self.ws, 0


class HostRuntime:
    def __init__(self, tag: str):
        self.tag = tag
        self.registry = {}
        self.n_buffers = 0

    compute = staticmethod(lambda dev: None)
    comm = staticmethod(lambda dev: None)
    copy_streams = staticmethod(lambda dev, n: [None] * n)
    on = staticmethod(lambda s: _Null())
    record = staticmethod(lambda s: None)
    wait = staticmethod(lambda s, ev: None)
    join = staticmethod(lambda s, other: None)
    host_wait = staticmethod(lambda ev: None)
    keep = staticmethod(lambda t, s: None)

    @staticmethod
    def host_buffer(n, dtype):
        return torch.empty(n, dtype=dtype)

    def buffers(self, group, rank, world_size, dev):
        self.n_buffers += 1
        return ShmBuffers(group, rank, world_size, f"{self.tag}b{self.n_buffers}", self.registry)

    def view(self, ptr, shape, dtype, dev):
        base = max(b for b in self.registry if b <= ptr)
        shm = self.registry[base]
        n = int(np.prod(shape))
        return torch.frombuffer(shm.buf, dtype=dtype, count=n, offset=ptr - base).view(*shape)

    @staticmethod
    def copy(segs, s):
        for dst, src, n in segs:
            if n > 0:
                ctypes.memmove(dst, src, n)
