"""Tensor parallelism over d_inner for MambaModel (one process per GPU, torch.distributed).

Each rank holds a contiguous 1/world slice of every layer's inner channels:

- in_proj  : the x-half rows and the z-half rows of its channel slice (column-parallel);
- conv1d, dt_proj (weight rows + bias), A_log, D: its channel slice;
- x_proj   : the columns of its channel slice (row-parallel) -> partial (B, dt_rank + 2N), all-reduced;
- out_proj : the columns of its channel slice (row-parallel) -> partial (B, d_model), all-reduced;
- embeddings, RMSNorm weights and the tied head: replicated.

Mamba-1's x_proj reads every inner channel, so a layer needs two all-reduces (after x_proj and after
out_proj); the scan, the conv and the decode step themselves need no communication. The partial sums are
reduced in float32. The reference has no multi-device code; this is the configs[3] layout of the
B200 build.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from mamba_metal_b200.mamba_block import decode_linear
from mamba_metal_b200.mamba_model import MambaConfig, MambaModel


def channel_range(d_inner: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous inner-channel slice [lo, hi) of `rank` (d_inner must divide evenly)."""
    if d_inner % world:
        raise ValueError(f"d_inner {d_inner} is not divisible by the tensor-parallel size {world}")
    per = d_inner // world
    return rank * per, (rank + 1) * per


def shard_state_dict(sd: dict, cfg: MambaConfig, rank: int, world: int) -> dict:
    """Slices a full MambaModel state_dict for one tensor-parallel rank (pure tensor indexing)."""
    d_inner = cfg.expand * cfg.d_model
    lo, hi = channel_range(d_inner, rank, world)
    out = {}
    for k, v in sd.items():
        if ".mixer." not in k:
            out[k] = v
            continue
        name = k.split(".mixer.", 1)[1]
        if name == "in_proj.weight":
            out[k] = torch.cat([v[lo:hi], v[d_inner + lo:d_inner + hi]], dim=0)
        elif name in ("conv1d.weight", "conv1d.bias", "dt_proj.weight", "dt_proj.bias", "A_log", "D"):
            out[k] = v[lo:hi]
        elif name in ("x_proj.weight", "out_proj.weight"):
            out[k] = v[:, lo:hi]
        else:
            raise KeyError(k)
    return {k: v.contiguous() for k, v in out.items()}


class _TPProject:
    """Row-parallel projection + all-reduce. Decode-sized partials (at most `max_rows` rows) are written
    straight into their call site's peer-memory slot and summed by the library's peer all-reduce
    kernel; larger ones (prefill) are reduced by NCCL in float32."""

    def __init__(self, group, peer=None, max_rows: int = 0):
        self.group = group
        self.peer = peer
        self.max_rows = max_rows

    def __call__(self, x: torch.Tensor, w: torch.Tensor, site: int) -> torch.Tensor:
        rows = x.numel() // x.shape[-1]
        n = rows * w.shape[0]
        peer = self.peer
        if peer is not None and rows <= self.max_rows and x.dtype == peer.dtype and n <= peer.capacity[site]:
            part = peer.slot(site)[:n].view(rows, w.shape[0])
            decode_linear(x.reshape(rows, x.shape[-1]), w, out=part)
            out = torch.empty((rows, w.shape[0]), dtype=x.dtype, device=x.device)
            peer.reduce(site, n, out)
            return out.view(*x.shape[:-1], w.shape[0])
        t32 = F.linear(x, w).float()
        dist.all_reduce(t32, group=self.group)
        return t32.to(x.dtype)

    def transposed(self, w: torch.Tensor, x_t: torch.Tensor, site: int) -> torch.Tensor:
        """w @ x_t for a (K, tokens) activation (the channel-first prefill), all-reduced by NCCL in float32."""
        t32 = torch.matmul(w, x_t).float()
        dist.all_reduce(t32, group=self.group)
        return t32.to(x_t.dtype)

    def partial(self, x: torch.Tensor, w: torch.Tensor, site: int):
        """Writes this rank's x @ w.T into the site's peer slot and returns a _PendingReduce whose
        add_rmsnorm finishes the all-reduce fused with the next residual add + RMSNorm; None when the
        call does not take the peer path (then the caller reduces as usual)."""
        rows = x.numel() // x.shape[-1]
        n = rows * w.shape[0]
        peer = self.peer
        if peer is None or rows > self.max_rows or x.dtype != peer.dtype or n > peer.capacity[site] \
                or n * peer.esize > peer.ll_max_bytes:
            return None
        part = peer.slot(site)[:n].view(rows, w.shape[0])
        decode_linear(x.reshape(rows, x.shape[-1]), w, out=part)
        return _PendingReduce(peer, site, rows, w.shape[0])


class _PendingReduce:
    """An out_proj partial already in its peer slot, reduced by the next pre-norm (mamba_model.py:49-58)."""

    def __init__(self, peer, site: int, rows: int, dim: int):
        self.peer, self.site, self.rows, self.dim = peer, site, rows, dim

    def add_rmsnorm(self, residual: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype: torch.dtype):
        out = torch.empty(residual.shape, dtype=out_dtype, device=residual.device)
        return self.peer.reduce_add_rmsnorm(self.site, self.rows, self.dim, residual, weight, eps, out)


def tp_model(full: MambaModel, rank: int, world: int, group=None, peer_rows: int = 0) -> MambaModel:
    """Builds this rank's tensor-parallel MambaModel from a full one (same device and dtype).

    The returned model holds the local channel slice in every mixer and all-reduces after x_proj and
    after out_proj; its forward / prefill / step / generation API is unchanged (conv and SSM states
    are per-rank slices of d_inner). With peer_rows > 0, projections of up to that many rows (decode
    batches) reduce through NVLink peer memory instead of NCCL."""
    cfg = full.cfg
    dev = full.embeddings.weight.device
    sd = shard_state_dict(full.state_dict(), cfg, rank, world)
    with torch.device("meta"):
        local = MambaModel(cfg, dtype=full.dtype, tp_world=world)
    local = local.to_empty(device=dev)
    local.load_state_dict(sd, strict=True)
    peer = None
    if peer_rows > 0 and world > 1:
        from mamba_metal_b200.comm import PeerAllReduce

        dt_rank = local.layers[0].mixer.dt_rank
        sites = []
        for _ in local.layers:
            sites += [peer_rows * (dt_rank + 2 * cfg.d_state), peer_rows * cfg.d_model]
        peer = PeerAllReduce(group if group is not None else dist.group.WORLD, dev, full.dtype, sites)
    proj = _TPProject(group, peer, peer_rows)
    for i, layer in enumerate(local.layers):
        layer.mixer.tp_reduce = proj
        layer.mixer.tp_sites = (2 * i, 2 * i + 1)
    local.tp_peer = peer
    return local
