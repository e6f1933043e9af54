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

    ``slot_numels[i]`` is the largest partial (in elements) call site i will reduce. Each site owns a
    receive area of ``world`` partials in one symmetric buffer; a producer writes this rank's partial
    straight into ``slot(i)`` (e.g. as a GEMM output) and ``reduce(i, n, out)`` sums the n-element
    partials of every rank into ``out``. Peers rewrite a site's area as soon as they have passed the
    previous call, so consecutive calls must use different sites; all ranks must make the same sequence
    of calls.
    """

    THREADS = 256  # the kernel's CTA size

    def __init__(self, group, device, dtype: torch.dtype, slot_numels: list[int], ll_max_bytes: int = 1 << 20):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MM_MAX_TP:
            raise ValueError(f"peer all-reduce supports up to {_lib.MM_MAX_TP} ranks")
        self.dtype = dtype
        self.device = torch.device(device)
        esize = torch.tensor([], dtype=dtype).element_size()
        gran = 256 // esize  # regions start on 256-byte boundaries
        self.ll_max_bytes = int(ll_max_bytes)
        self.offsets, self.capacity, self.strides = [], [], []
        total = 0
        for n in slot_numels:
            stride = 2 * ((int(n) + gran - 1) // gran * gran)  # room for the low-latency lines
            self.offsets.append(total)
            self.capacity.append(int(n))
            self.strides.append(stride)
            total += self.world * stride
        self.buf = symm_mem.empty(max(total, gran), dtype=dtype, device=self.device)
        h = symm_mem.rendezvous(self.buf, group)
        self.buf_ptrs = [int(x) for x in h.buffer_ptrs]
        self.buf.zero_()
        self.sig = symm_mem.empty(_lib.MM_PEER_MAX_BLOCKS * _lib.MM_MAX_TP, dtype=torch.int32, device=self.device)
        self.sig.zero_()
        hs = symm_mem.rendezvous(self.sig, group)
        self.sig_ptrs = [int(x) for x in hs.buffer_ptrs]
        self.counters = torch.zeros(_lib.MM_PEER_MAX_BLOCKS + 3, dtype=torch.int32, device=self.device)
        self.esize = esize
        self.vec = 16 // esize
        torch.cuda.synchronize(self.device)
        dist.barrier(group)

    def slot(self, site: int) -> torch.Tensor:
        """This rank's partial of call site `site` (capacity elements)."""
        off = self.offsets[site] + self.rank * self.strides[site]
        return self.buf[off:off + self.capacity[site]]

    def protocol(self, n: int) -> int:
        """Low-latency lines up to ll_max_bytes of partial, the flag protocol above."""
        return _lib.MM_PEER_LL if n * self.esize <= self.ll_max_bytes else _lib.MM_PEER_FLAGS

    def blocks(self, n: int, protocol: int) -> int:
        """CTAs for an n-element call: about two 16-byte vectors (flags) or two 8-byte lines (LL) per
        thread, at most MM_PEER_MAX_BLOCKS."""
        per_cta = self.THREADS * 2 * (self.vec if protocol == _lib.MM_PEER_FLAGS else 8 // self.esize)
        return max(1, min(_lib.MM_PEER_MAX_BLOCKS, -(-n // per_cta)))

    def _args(self, site: int, n: int, proto: int) -> "_lib.MMPeerReduceArgs":
        if n > self.capacity[site]:
            raise ValueError("partial larger than its slot")
        a = _lib.MMPeerReduceArgs()
        off = self.offsets[site] * self.esize
        for r in range(self.world):
            a.slots[r] = self.buf_ptrs[r] + off
            a.signals[r] = self.sig_ptrs[r]
        a.counters = self.counters.data_ptr()
        a.dtype = _lib.DTYPE_CODE[self.dtype]
        a.n, a.stride, a.world, a.rank = n, self.strides[site], self.world, self.rank
        a.nblocks, a.protocol = self.blocks(n, proto), proto
        return a

    def reduce(self, site: int, n: int, out: torch.Tensor) -> torch.Tensor:
        a = self._args(site, n, self.protocol(n))
        a.out = out.data_ptr()
        with torch.cuda.device(self.device):
            rc = _lib.lib().mm_peer_allreduce(ctypes.byref(a), _lib.stream_handle(self.device))
        _lib.check(rc, "mm_peer_allreduce")
        return out

    def reduce_add_rmsnorm(self, site: int, rows: int, dim: int, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float, out: torch.Tensor) -> torch.Tensor:
        """Sums the (rows, dim) partials of site `site` (low-latency protocol), adds the sum (rounded to the
        buffer dtype) into the fp32 `residual` in place and writes RMSNorm(residual) * weight to `out`."""
        assert residual.is_contiguous() and residual.dtype == torch.float32 and residual.numel() == rows * dim
        assert weight.dtype == torch.float32 and out.dtype == self.dtype and out.is_contiguous()
        a = _lib.MMPeerAddNormArgs()
        a.reduce = self._args(site, rows * dim, _lib.MM_PEER_LL)
        a.residual, a.weight, a.out = residual.data_ptr(), weight.data_ptr(), out.data_ptr()
        a.rows, a.dim, a.out_stride_r, a.eps = rows, dim, dim, float(eps)
        with torch.cuda.device(self.device):
            rc = _lib.lib().mm_peer_allreduce_add_rmsnorm(ctypes.byref(a), _lib.stream_handle(self.device))
        _lib.check(rc, "mm_peer_allreduce_add_rmsnorm")
        return out

    def timed_out(self) -> bool:
        """True if any wait gave up (a peer never arrived); synchronises the device."""
        return bool(self.counters[_lib.MM_PEER_MAX_BLOCKS].item())
