"""Tensor-parallel model over 2 GPUs (NCCL) against the same model on one GPU. Needs >= 2 GPUs; skipped
otherwise. Each rank runs in its own spawned process; failures are reported through a queue."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, peer_rows=0):
    import datetime

    import torch.distributed as dist

    from mamba_metal_b200 import MambaConfig, MambaModel, generate_ids, init_weights_
    from mamba_metal_b200.parallel import tp_model

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        cfg = MambaConfig(d_model=256, n_layer=3, vocab_size=997, dt_rank=16)
        full = init_weights_(MambaModel(cfg, device=dev), seed=7)
        ids = torch.randint(0, cfg.vocab_size, (4, 37), generator=torch.Generator().manual_seed(2)).to(dev)
        with torch.no_grad():
            ref_logits = full(ids)
            _, ref_conv, ref_ssm = full.prefill(ids)
            ref_out = generate_ids(full, ids, 8)
            tp = tp_model(full, rank, world, peer_rows=peer_rows)
            logits = tp(ids)
            _, conv, ssm = tp.prefill(ids)
            out = generate_ids(tp, ids, 8)
        lo = rank * tp.d_inner
        ok_logits = torch.allclose(logits, ref_logits, rtol=1e-4, atol=1e-4 * float(ref_logits.abs().mean()))
        ok_state = torch.allclose(ssm[1], ref_ssm[1][:, lo:lo + tp.d_inner], rtol=1e-4, atol=1e-5)
        ok_conv = torch.allclose(conv[2], ref_conv[2][:, lo:lo + tp.d_inner], rtol=1e-5, atol=1e-6)
        same_tokens = bool(torch.equal(out, ref_out))
        if tp.tp_peer is not None:
            assert not tp.tp_peer.timed_out()
        q.put((rank, ok_logits, ok_state, ok_conv, same_tokens, float((logits - ref_logits).abs().max())))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, False, False, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("peer_rows", [0, 64])
def test_tp2_matches_single_gpu(peer_rows):
    """NCCL reductions (peer_rows=0) and the NVLink peer all-reduce for decode-sized projections."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, peer_rows)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] and r[2] and r[3] and r[4] for r in res), res


def _peer_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from mamba_metal_b200.comm import PeerAllReduce

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        sizes = [1, 7, 100, 12288, 163843]
        bad = []
        for dtype, ll_max in ((torch.float32, 1 << 16), (torch.bfloat16, 1 << 16), (torch.bfloat16, 0),
                              (torch.float16, 1 << 30)):
            peer = PeerAllReduce(dist.group.WORLD, dev, dtype, sizes, ll_max_bytes=ll_max)
            for it in range(3):
                for site, n in enumerate(sizes):
                    parts = [torch.randn(n, generator=torch.Generator().manual_seed(1000 * it + 10 * site + r))
                             .to(dtype) for r in range(world)]
                    peer.slot(site)[:n].copy_(parts[rank])
                    out = torch.empty(n, dtype=dtype, device=dev)
                    peer.reduce(site, n, out)
                    want = parts[0].float()
                    for r in range(1, world):
                        want = want + parts[r].float()
                    if not torch.equal(out.cpu(), want.to(dtype)):
                        bad.append((str(dtype), ll_max, it, n))
            if peer.timed_out():
                bad.append((str(dtype), "timeout"))
            del peer
        # all-reduce fused with residual add + RMSNorm (low-latency protocol, one CTA per row)
        for dtype in (torch.float32, torch.bfloat16):
            rows, dim = 5, 2560
            peer = PeerAllReduce(dist.group.WORLD, dev, dtype, [rows * dim, rows * dim])
            g = torch.Generator().manual_seed(77)
            res0 = torch.randn(rows, dim, generator=g)
            w = torch.rand(dim, generator=g) + 0.5
            for it in range(3):
                parts = [torch.randn(rows, dim, generator=torch.Generator().manual_seed(500 + 10 * it + r)).to(dtype)
                         for r in range(world)]
                site = it % 2
                peer.slot(site)[:rows * dim].view(rows, dim).copy_(parts[rank])
                res = res0.to(dev).contiguous()
                out = torch.empty(rows, dim, dtype=dtype, device=dev)
                peer.reduce_add_rmsnorm(site, rows, dim, res, w.to(dev), 1e-5, out)
                s = parts[0].float()
                for r in range(1, world):
                    s = s + parts[r].float()
                want_res = res0 + s.to(dtype).float()
                want = want_res * torch.rsqrt((want_res * want_res).mean(-1, keepdim=True) + 1e-5) * w
                if not torch.equal(res.cpu(), want_res):
                    bad.append(("addnorm residual", str(dtype), it))
                tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
                if not torch.allclose(out.float().cpu(), want.to(dtype).float(), rtol=tol, atol=tol):
                    bad.append(("addnorm out", str(dtype), it))
            if peer.timed_out():
                bad.append((str(dtype), "addnorm timeout"))
            del peer
        q.put((rank, bad))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, [repr(e)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_exact():
    """mm_peer_allreduce on 2 GPUs: ragged and vector sizes, fp32 / bf16 / fp16, both protocols (flags,
    low-latency lines) and the size-based mix, sites used in rotation; the result equals the rank-ordered
    fp32 sum rounded to the buffer type, bit for bit."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(not r[1] for r in res), res


def _fused_dt_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import mamba_metal_b200.mamba_block as mb
    from mamba_metal_b200 import MambaConfig, MambaModel, init_weights_
    from mamba_metal_b200.parallel import tp_model

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = MambaConfig(d_model=256, n_layer=2, vocab_size=997, dt_rank=16)
        full = init_weights_(MambaModel(cfg, dtype=torch.bfloat16, device=dev), seed=7)
        ids = torch.randint(0, cfg.vocab_size, (8, 29), generator=torch.Generator().manual_seed(4)).to(dev)
        tp = tp_model(full, rank, world, peer_rows=64)
        default = mb.FUSED_DT_STEP
        mb.FUSED_DT_STEP = True
        applies = all(layer.mixer._fused_dt_step(ids.shape[0]) for layer in tp.layers)
        outs = {}
        with torch.no_grad():
            _, conv, ssm = tp.prefill(ids)
            for fused in (False, True):
                mb.FUSED_DT_STEP = fused
                logits, _, ssm2 = tp.step(ids[:, -1:], [c.clone() for c in conv], [s.clone() for s in ssm])
                outs[fused] = (logits.float(), ssm2[-1].clone())
        mb.FUSED_DT_STEP = default
        rel = lambda a, b: float((a - b).norm() / b.norm())
        q.put((rank, applies, rel(outs[True][0], outs[False][0]), rel(outs[True][1], outs[False][1])))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_fused_dt_step_matches_dt_gemm():
    """bf16 tensor-parallel decode step: dt_proj computed inside the SSM step kernel (from the all-reduced
    x_proj output and this rank's dt_proj rows) against dt_proj as a separate GEMM. The GEMM rounds dt to
    bf16 and the fused step does not, so the two agree to bf16 accuracy (relative L2 <= 1e-2)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_dt_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] is True and r[2] < 1e-2 and r[3] < 1e-2 for r in res), res
