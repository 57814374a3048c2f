"""Peer-memory exchange region for Ulysses sequence parallelism on one node.

Every rank allocates one region with the same layout (the head-sharded q
buffer, the attention output buffer of its tokens and every layer's
[current | cache] K/V buffers), exports its CUDA IPC handle and opens the
others' (legacy CUDA IPC through the C ABI: plain peer-to-peer mappings, no
NVLink multicast objects).  The QKV projection's epilogue
(jo_fp8_scaled_mm_scatter) then stores each (token, head) straight into the
owning rank's region over NVLink, which replaces the all-to-all that turns the
token shard into a head shard; the attention epilogue
(jo_attention_fwd_scatter) stores each output row back into the region of the
rank that owns the token, which replaces the all-to-all after attention.

Ordering: a rank reads its region only after a one-element NCCL all-reduce
that every rank enqueues after its scatters (sync()), once after the QKV
projections and once after attention; the second also keeps a faster rank's
next-layer scatters from overwriting the q buffer a slower rank's attention
still reads.  The same call after the KV-cache commit keeps the next chunk's
scatters from overtaking the commit copies of a slower rank.
"""
from __future__ import annotations

import ctypes
from typing import List

import torch

from joyomni_ops import _lib

_ALIGN = 256


class RegionLayout:
    """Byte offsets of named buffers inside the region (256-byte aligned)."""

    def __init__(self):
        self.size = 0
        self.entries = {}

    def add(self, name: str, shape, dtype=torch.bfloat16) -> int:
        off = (self.size + _ALIGN - 1) // _ALIGN * _ALIGN
        n = 1
        for d in shape:
            n *= int(d)
        self.entries[name] = (off, tuple(int(d) for d in shape), dtype)
        self.size = off + n * torch.empty((), dtype=dtype).element_size()
        return off

    def offset(self, name: str) -> int:
        return self.entries[name][0]


class LocalRegion:
    """The same layout in one local allocation (a single rank: nothing to map)."""

    def __init__(self, layout: RegionLayout, device):
        self.layout = layout
        self.local = torch.empty(layout.size, dtype=torch.uint8, device=device)

    def tensor(self, name: str) -> torch.Tensor:
        return PeerRegion.tensor(self, name)

    def ptr(self, rank: int, name: str) -> int:
        assert rank == 0
        return self.local.data_ptr() + self.layout.offset(name)

    def sync(self) -> None:
        pass

    def close(self) -> None:
        pass


class PeerRegion:
    def __init__(self, layout: RegionLayout, group, world: int, rank: int, device):
        import torch.distributed as dist
        self.layout = layout
        self.group = group
        self.world = world
        self.rank = rank
        self.local = torch.empty(layout.size, dtype=torch.uint8, device=device)
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_int64(0)
        _lib.check(_lib.lib.jo_ipc_get_handle(self.local.data_ptr(), handle, ctypes.byref(off)))
        mine = (bytes(handle.raw), int(off.value), int(layout.size))
        every: List = [None] * world
        dist.all_gather_object(every, mine, group=group)
        if any(e[2] != layout.size for e in every):
            raise RuntimeError("peer exchange regions differ in size across ranks")
        self.bases: List[int] = []
        self._opened: List[int] = []
        for r, (hb, o, _) in enumerate(every):
            if r == rank:
                self.bases.append(self.local.data_ptr())
                continue
            p = ctypes.c_void_p()
            _lib.check(_lib.lib.jo_ipc_open(hb, ctypes.byref(p)))
            self._opened.append(p.value)
            self.bases.append(p.value + o)
        self._flag = torch.zeros(1, dtype=torch.float32, device=device)

    def tensor(self, name: str) -> torch.Tensor:
        """This rank's buffer `name` as a tensor view of the region."""
        off, shape, dtype = self.layout.entries[name]
        n = 1
        for d in shape:
            n *= d
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return self.local[off:off + nbytes].view(dtype).view(shape)

    def ptr(self, rank: int, name: str) -> int:
        """Device address of rank `rank`'s buffer `name` (a peer mapping for other ranks)."""
        return self.bases[rank] + self.layout.offset(name)

    def sync(self) -> None:
        """Stream-ordered cross-rank synchronisation (one-element all-reduce)."""
        import torch.distributed as dist
        dist.all_reduce(self._flag, group=self.group)

    def close(self, barrier: bool = True) -> None:
        """Unmap the peers' regions, after a barrier so that no rank still
        writes (barrier=False: the caller has synchronised every rank)."""
        import torch.distributed as dist
        if barrier:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        for p in self._opened:
            _lib.check(_lib.lib.jo_ipc_close(p))
        self._opened = []
