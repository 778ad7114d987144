"""Sharding the fused CorrVolume -> CostStem3D op over several GPUs.

One process per GPU (``torch.distributed``; NCCL over NVLink on GPUs, gloo
on CPU for the host-logic tests).  Two partitions, neither with a collective
inside the op:

* batch -- rank k takes batch items ``split_even(B, world, k)``; no exchange
  at all (the stereo pairs are independent).
* rows  -- one image pair split by image rows.  Rank k owns feature rows
  ``[r0, r1) = split_even(H, world, k)`` and produces output rows
  ``[r0, r1)``.  Correlation is row-local and the stem reaches one row up and
  one down, so a rank needs exactly one extra feature row from each
  neighbour.  ``exchange_halo`` fetches them by point-to-point send/recv
  before the local ``corr_cost_stem3d_band`` call; the stitched output is
  identical to the unsharded call.

The per-rank computation defaults to the CUDA op
(``whirlwind_trt_plugins_b200.corr_cost_stem3d_band``); ``band_fn`` lets a
caller substitute another implementation with the same signature.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["split_even", "halo_rows", "exchange_halo", "HaloBand", "corr_cost_stem3d_rows",
           "corr_cost_stem3d_batch", "gather_rows"]


def split_even(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's share of n items; the first n % world ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank outside the world")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def halo_rows(H: int, r0: int, r1: int) -> tuple[int, int]:
    """Feature rows a rank producing output rows [r0, r1) must hold."""
    return max(0, r0 - 1), min(H, r1 + 1)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _peer(group, rank_in_group: int) -> int:
    """Global rank of a group member (send/recv take global ranks)."""
    return rank_in_group if group is None else dist.get_global_rank(group, rank_in_group)


def exchange_halo(x_local: torch.Tensor, H: int, group=None) -> tuple[torch.Tensor, int]:
    """Extend this rank's feature rows by one row from each neighbour.

    x_local: [B, C, r1 - r0, W], this rank's rows of an H-row image (row split
    of ``split_even``).  Returns (band, i0): band holds rows [i0, i1) of
    ``halo_rows(H, r0, r1)``.  Every rank must call this; all ranks post their
    sends and receives in one batch, so the order cannot deadlock."""
    world, rank = _world(group)
    r0, r1 = split_even(H, world, rank)
    if x_local.dim() != 4 or x_local.shape[2] != r1 - r0:
        raise ValueError(f"rank {rank}: expected rows [{r0}, {r1}) of an {H}-row image, "
                         f"got shape {tuple(x_local.shape)}")
    if H < world:
        raise ValueError("row sharding needs at least one image row per rank")
    B, C, _, W = x_local.shape
    i0, i1 = halo_rows(H, r0, r1)
    band = x_local.new_empty((B, C, i1 - i0, W))
    band[:, :, r0 - i0:r1 - i0].copy_(x_local)
    ops = []
    top = bot = None
    if rank > 0:
        top = x_local.new_empty((B, C, 1, W))
        ops.append(dist.P2POp(dist.isend, x_local[:, :, :1].contiguous(), _peer(group, rank - 1), group))
        ops.append(dist.P2POp(dist.irecv, top, _peer(group, rank - 1), group))
    if rank < world - 1:
        bot = x_local.new_empty((B, C, 1, W))
        ops.append(dist.P2POp(dist.isend, x_local[:, :, -1:].contiguous(), _peer(group, rank + 1), group))
        ops.append(dist.P2POp(dist.irecv, bot, _peer(group, rank + 1), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if top is not None:
        band[:, :, :1].copy_(top)
    if bot is not None:
        band[:, :, -1:].copy_(bot)
    return band, i0


class HaloBand:
    """A rank's persistent row band of one feature map, for repeated
    row-sharded calls: ``band`` [B, C, i1 - i0, W] holds image rows
    [i0, i1) = ``halo_rows(H, r0, r1)``; the caller (e.g. the feature network)
    writes its own rows [r0, r1) into ``own`` once per frame, and
    ``exchange()`` fetches only the two halo rows from the neighbours (one
    contiguous [B, C, 1, W] message per side and direction) and writes them
    into the band's edge rows.  Nothing is allocated per call."""

    def __init__(self, B: int, C: int, H: int, W: int, dtype, device, group=None):
        world, rank = _world(group)
        if H < world:
            raise ValueError("row sharding needs at least one image row per rank")
        self.group, self.world, self.rank, self.H = group, world, rank, H
        self.r0, self.r1 = split_even(H, world, rank)
        self.i0, self.i1 = halo_rows(H, self.r0, self.r1)
        self.band = torch.zeros((B, C, self.i1 - self.i0, W), dtype=dtype, device=device)
        self.own = self.band[:, :, self.r0 - self.i0:self.r1 - self.i0]
        row = (B, C, 1, W)
        self._send_top = torch.empty(row, dtype=dtype, device=device) if rank > 0 else None
        self._recv_top = torch.empty(row, dtype=dtype, device=device) if rank > 0 else None
        self._send_bot = torch.empty(row, dtype=dtype, device=device) if rank < world - 1 else None
        self._recv_bot = torch.empty(row, dtype=dtype, device=device) if rank < world - 1 else None

    def exchange(self) -> None:
        ops = []
        k0 = self.r0 - self.i0  # band index of the first own row
        k1 = self.r1 - self.i0  # one past the last own row
        if self._send_top is not None:
            self._send_top.copy_(self.band[:, :, k0:k0 + 1])
            peer = _peer(self.group, self.rank - 1)
            ops.append(dist.P2POp(dist.isend, self._send_top, peer, self.group))
            ops.append(dist.P2POp(dist.irecv, self._recv_top, peer, self.group))
        if self._send_bot is not None:
            self._send_bot.copy_(self.band[:, :, k1 - 1:k1])
            peer = _peer(self.group, self.rank + 1)
            ops.append(dist.P2POp(dist.isend, self._send_bot, peer, self.group))
            ops.append(dist.P2POp(dist.irecv, self._recv_bot, peer, self.group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        if self._recv_top is not None:
            self.band[:, :, :1].copy_(self._recv_top)
        if self._recv_bot is not None:
            self.band[:, :, -1:].copy_(self._recv_bot)


def _default_band_fn():
    from . import corr_cost_stem3d_band
    return corr_cost_stem3d_band


def corr_cost_stem3d_rows(left_local, right_local, w, b, max_disp: int, num_groups: int, H: int,
                          act: int = 0, group=None, band_fn=None):
    """Row-sharded fused op: returns this rank's output rows [B, Cout, D, r1 - r0, W]."""
    world, rank = _world(group)
    r0, r1 = split_even(H, world, rank)
    lb, i0 = exchange_halo(left_local, H, group)
    rb, _ = exchange_halo(right_local, H, group)
    fn = band_fn or _default_band_fn()
    return fn(lb, rb, w, b, max_disp, num_groups, H, i0, r0, r1 - r0, act)


def corr_cost_stem3d_batch(left, right, w, b, max_disp: int, num_groups: int, act: int = 0, group=None):
    """Batch-sharded fused op over the full batch held by every rank: rank k
    computes batch items split_even(B, world, k) and returns that slice."""
    from . import corr_cost_stem3d
    world, rank = _world(group)
    b0, b1 = split_even(left.shape[0], world, rank)
    if b1 == b0:
        Cout = b.numel()
        return left.new_empty((0, Cout, max_disp) + tuple(left.shape[2:]))
    return corr_cost_stem3d(left[b0:b1].contiguous(), right[b0:b1].contiguous(), w, b, max_disp,
                            num_groups, act)


def gather_rows(out_local: torch.Tensor, H: int, group=None) -> torch.Tensor:
    """All-gather the row shards [B, Cout, D, rows_k, W] into [B, Cout, D, H, W]
    on every rank (a convenience for callers that need the whole volume)."""
    world, rank = _world(group)
    rows = max(split_even(H, world, k)[1] - split_even(H, world, k)[0] for k in range(world))
    pad = out_local.new_zeros(out_local.shape[:3] + (rows,) + out_local.shape[4:])
    pad[:, :, :, :out_local.shape[3]].copy_(out_local)
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous(), group=group)
    pieces = []
    for k in range(world):
        r0, r1 = split_even(H, world, k)
        pieces.append(parts[k][:, :, :, :r1 - r0])
    return torch.cat(pieces, dim=3)
