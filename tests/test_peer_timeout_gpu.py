"""The peer all-reduce's waits are bounded: with a peer that never arrives, each protocol gives up after
its 2 s limit, sets the error word, finishes the launch and leaves the context usable. One GPU: "rank 1"
is played by local buffers that nothing writes (a flag that nothing sets); no kernel waits on another
kernel, and nothing faults."""

import ctypes
import time

import pytest
import torch

from mamba_metal_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("protocol", [_lib.MM_PEER_FLAGS, _lib.MM_PEER_LL])
def test_missing_peer_times_out(protocol):
    n, stride = 1000, 2048  # stride: room for the LL lines of n bf16 elements
    area0 = torch.zeros(2 * stride, dtype=torch.bfloat16, device=DEV)    # this rank's receive area
    area1 = torch.zeros(2 * stride, dtype=torch.bfloat16, device=DEV)    # stands in for the peer's
    sig0 = torch.zeros(_lib.MM_PEER_MAX_BLOCKS * _lib.MM_MAX_TP, dtype=torch.int32, device=DEV)
    sig1 = torch.zeros_like(sig0)
    counters = torch.zeros(_lib.MM_PEER_MAX_BLOCKS + 3, dtype=torch.int32, device=DEV)
    area0[:n] = 1.0  # this rank's partial
    out = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    a = _lib.MMPeerReduceArgs()
    a.slots[0], a.slots[1] = area0.data_ptr(), area1.data_ptr()
    a.signals[0], a.signals[1] = sig0.data_ptr(), sig1.data_ptr()
    a.counters, a.out = counters.data_ptr(), out.data_ptr()
    a.dtype, a.n, a.stride, a.world, a.rank, a.nblocks, a.protocol = _lib.MM_BF16, n, stride, 2, 0, 2, protocol
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.device(0):
        rc = _lib.lib().mm_peer_allreduce(ctypes.byref(a), _lib.stream_handle(torch.device(DEV)))
    assert rc == 0, _lib.ERROR_NAMES.get(rc, rc)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert counters[_lib.MM_PEER_MAX_BLOCKS].item() == 1, "the wait limit must set the error word"
    assert 1.5 < waited < 30, waited
    # the context is still usable
    x = torch.arange(10, device=DEV)
    assert int(x.sum()) == 45
