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


def _project_worker(rank, world, port, result_q):
    """tp_model's wiring and _TPProject (the NCCL/gloo path: no peer memory) on CPU tensors."""
    from mamba_metal_b200.parallel import _TPProject, tp_model

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = MambaConfig(d_model=32, n_layer=3, vocab_size=53, dt_rank=4)
        full = init_weights_(MambaModel(cfg), seed=5)
        local = tp_model(full, rank, world)
        E = cfg.expand * cfg.d_model
        lo, hi = channel_range(E, rank, world)
        g = torch.Generator().manual_seed(11)
        errs, ok = [], local.tp_peer is None and local.d_inner == E // world
        for i, (lb, fb) in enumerate(zip(local.layers, full.layers)):
            lm, fm = lb.mixer, fb.mixer
            ok &= isinstance(lm.tp_reduce, _TPProject) and lm.tp_sites == (2 * i, 2 * i + 1)
            xc = torch.randn(2, 9, E, generator=g)
            y = torch.randn(2, 9, E, generator=g)
            # row-parallel x_proj / out_proj: this rank's channel slice, all-reduced, equals the full product
            want_x = xc @ fm.x_proj.weight.T
            got_x = lm._project(xc[..., lo:hi], lm.x_proj.weight, 0)
            got_x2 = lm._project(xc[0, :, lo:hi], lm.x_proj.weight, 0)  # 2-D (decode-shaped) call
            want_o = y @ fm.out_proj.weight.T
            got_o = lm._project(y[..., lo:hi], lm.out_proj.weight, 1)
            # channel-first prefill form: W_x @ xc^T on (channels, tokens)
            xt = xc.reshape(-1, E).T.contiguous()
            got_t = lm._project_t(lm.x_proj.weight, xt[lo:hi], 0)
            want_t = fm.x_proj.weight @ xt
            # without peer memory the fused out_proj reduction is not taken
            ok &= lm.tp_reduce.partial(y[0, :, lo:hi], lm.out_proj.weight, lm.tp_sites[1]) is None
            for got, want in ((got_x, want_x), (got_x2, want_x[0]), (got_o, want_o), (got_t, want_t)):
                ok &= got.shape == want.shape and torch.allclose(got, want, rtol=1e-5, atol=1e-5)
                errs.append(float((got - want).abs().max()))
        result_q.put((rank, bool(ok), max(errs)))
    except Exception as e:  # pragma: no cover - reported to the parent
        result_q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tp_project_and_model_wiring():
    """The repo's tensor-parallel projection wrapper (parallel.py _TPProject, reached through
    MambaBlock._project / _project_t) and tp_model's per-layer wiring, on 2 gloo ranks."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_project_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert all(ok for _, ok, _ in res), res
