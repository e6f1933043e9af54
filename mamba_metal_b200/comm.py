"""Peer-memory all-reduce for the tensor-parallel decode step (libmamba_b200's mm_peer_allreduce).

torch.distributed's symmetric memory provides the plumbing only: a buffer and a signal array that every
rank of the group maps, and their per-rank device addresses. The reduction itself -- epoch-stamped
signals, bounded waits, peer loads over NVLink and the fp32 sum -- is the library's kernel.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from mamba_metal_b200 import _lib


class PeerAllReduce:
    """All-reduce of small partial sums through NVLink peer memory.

    ``slot_numels[i]`` is the largest partial (in elements) call site i will reduce. Each site gets its
    own slot in one symmetric buffer; a producer writes its partial straight into ``slot(i)`` (e.g. as a
    GEMM output) and ``reduce(i, n, out)`` sums the n-element partials of every rank into ``out``.
    Sites reuse their slot only on their next call, and the kernel's barrier keeps ranks at most one call
    apart, so no slot is overwritten while a peer still reads it. All ranks must make the same sequence
    of calls.
    """

    def __init__(self, group, device, dtype: torch.dtype, slot_numels: list[int], nblocks: int = 16):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MM_MAX_TP:
            raise ValueError(f"peer all-reduce supports up to {_lib.MM_MAX_TP} ranks")
        self.dtype = dtype
        self.device = torch.device(device)
        self.nblocks = int(nblocks)
        esize = torch.tensor([], dtype=dtype).element_size()
        gran = 256 // esize  # slots start on 256-byte boundaries
        self.offsets, self.capacity = [], []
        total = 0
        for n in slot_numels:
            self.offsets.append(total)
            self.capacity.append(int(n))
            total += (int(n) + gran - 1) // gran * gran
        self.buf = symm_mem.empty(max(total, gran), dtype=dtype, device=self.device)
        h = symm_mem.rendezvous(self.buf, group)
        self.buf_ptrs = [int(x) for x in h.buffer_ptrs]
        self.sig = symm_mem.empty(self.nblocks * _lib.MM_MAX_TP, dtype=torch.int32, device=self.device)
        self.sig.zero_()
        hs = symm_mem.rendezvous(self.sig, group)
        self.sig_ptrs = [int(x) for x in hs.buffer_ptrs]
        self.counters = torch.zeros(self.nblocks + 1, dtype=torch.int32, device=self.device)
        self.esize = esize
        torch.cuda.synchronize(self.device)
        dist.barrier(group)

    def slot(self, site: int) -> torch.Tensor:
        return self.buf[self.offsets[site]:self.offsets[site] + self.capacity[site]]

    def reduce(self, site: int, n: int, out: torch.Tensor) -> torch.Tensor:
        if n > self.capacity[site]:
            raise ValueError("partial larger than its slot")
        a = _lib.MMPeerReduceArgs()
        off = self.offsets[site] * self.esize
        for r in range(self.world):
            a.bufs[r] = self.buf_ptrs[r] + off
            a.signals[r] = self.sig_ptrs[r]
        a.counters = self.counters.data_ptr()
        a.out = out.data_ptr()
        a.dtype = _lib.DTYPE_CODE[self.dtype]
        a.n, a.world, a.rank, a.nblocks = n, self.world, self.rank, self.nblocks
        with torch.cuda.device(self.device):
            rc = _lib.lib().mm_peer_allreduce(ctypes.byref(a), _lib.stream_handle(self.device))
        _lib.check(rc, "mm_peer_allreduce")
        return out

    def timed_out(self) -> bool:
        """True if any wait gave up (a peer never arrived); synchronises the device."""
        return bool(self.counters[self.nblocks].item())
