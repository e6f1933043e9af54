"""Tensor-parallel sharding logic on CPU ranks (gloo, world size 2): the sharded projections plus the
all-reduce reproduce the unsharded block (oracle restatement, plain torch ops)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mamba_metal_b200 import MambaConfig, MambaModel, init_weights_
from mamba_metal_b200.parallel import channel_range, shard_state_dict
from oracle.model_ref import RefMixer, RefModel


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        cfg = MambaConfig(d_model=32, n_layer=2, vocab_size=53, dt_rank=4)
        full = init_weights_(MambaModel(cfg), seed=3)
        sd = {k: v.detach() for k, v in full.state_dict().items()}
        local = shard_state_dict(sd, cfg, rank, world)
        ref = RefModel(sd, cfg)
        x = torch.randn(2, 9, 32, generator=torch.Generator().manual_seed(1))
        # prefill of layer 0 with sharded weights + all-reduce after x_proj and out_proj
        m_full = RefMixer(sd, "layers.0.mixer.", cfg.d_state, cfg.dt_rank)
        m_loc = RefMixer(local, "layers.0.mixer.", cfg.d_state, cfg.dt_rank)
        E, N, R = m_loc.E, m_loc.N, m_loc.R
        xz = x @ m_loc.W_in.T
        xm, z = xz[..., :E], xz[..., E:]
        xc = torch.nn.functional.silu(m_loc._conv(xm))
        x_dbl = xc @ m_loc.W_x.T
        dist.all_reduce(x_dbl)
        dt = x_dbl[..., :R] @ m_loc.W_dt.T + m_loc.b_dt
        from oracle.model_ref import scan_seq

        y, h = scan_seq(xc.transpose(1, 2), dt.transpose(1, 2), m_loc.A, x_dbl[..., R:R + N].transpose(1, 2),
                        x_dbl[..., R + N:].transpose(1, 2), m_loc.D, z.transpose(1, 2))
        out = y.transpose(1, 2) @ m_loc.W_out.T
        dist.all_reduce(out)
        y_ref, _, h_ref = m_full.prefill(x)
        lo, hi = channel_range(2 * 32, rank, world)
        ok = torch.allclose(out, y_ref, rtol=1e-4, atol=1e-5) and torch.allclose(h, h_ref[:, lo:hi], rtol=1e-4,
                                                                                    atol=1e-6)
        result_q.put((rank, bool(ok), float((out - y_ref).abs().max())))
    finally:
        dist.destroy_process_group()


def test_tp_sharding_reproduces_full_block():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert all(ok for _, ok, _ in res), res


def test_shard_shapes_and_validation():
    cfg = MambaConfig(d_model=48, n_layer=1, vocab_size=17, dt_rank=3)
    sd = MambaModel(cfg).state_dict()
    loc = shard_state_dict(sd, cfg, 1, 4)
    assert loc["layers.0.mixer.in_proj.weight"].shape == (2 * 24, 48)
    assert loc["layers.0.mixer.x_proj.weight"].shape == (3 + 32, 24)
    assert loc["layers.0.mixer.out_proj.weight"].shape == (48, 24)
    assert loc["layers.0.mixer.conv1d.weight"].shape == (24, 1, 4)
    torch.testing.assert_close(loc["layers.0.mixer.in_proj.weight"][:24], sd["layers.0.mixer.in_proj.weight"][24:48])
    torch.testing.assert_close(loc["layers.0.mixer.in_proj.weight"][24:], sd["layers.0.mixer.in_proj.weight"][96 + 24:96 + 48])
    with pytest.raises(ValueError):
        channel_range(96, 0, 5)
    with torch.device("meta"):
        m = MambaModel(cfg, tp_world=4)
    assert m.layers[0].mixer.d_inner == 24 and m.d_inner == 24
