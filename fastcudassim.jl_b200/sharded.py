"""Batch sharding over the GPUs of one node (one process per GPU).

Images are independent (the reference loops over them, src/core.jl:186), so a
batch splits into contiguous slices with no exchange in the data path.  The
only communication is one all-gather of the per-image (D)SSIM scalars, so every
rank ends with the full vector while each rank's gradient slice stays resident
on its own GPU.  With the NCCL backend the all-gather runs over NVLink.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .interface import dssim_with_gradient_, ssim_with_gradient_


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of n images for `rank` (the first n % world ranks get one more)."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def gather_scores(local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather per-image scores of unequal shards into one length-n_total vector."""
    world = dist.get_world_size(group)
    per = -(-n_total // world)
    buf = torch.zeros(per, dtype=local.dtype, device=local.device)
    buf[: local.numel()].copy_(local)
    out = torch.empty(per * world, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    parts = []
    for r in range(world):
        lo, hi = shard_range(n_total, world, r)
        parts.append(out[r * per: r * per + (hi - lo)])
    return torch.cat(parts)


def sharded_with_gradient(imgs1_shard, imgs2_shard, n_total: int, dssim: bool = False,
                          divide_by_two_in_dssim: bool = False, ssims_shard=None, grad_shard=None,
                          group=None):
    """(D)SSIM with gradient on this rank's shard, then the all-gather of the scores.

    Returns ``(all_scores, grad_shard)``: the full length-``n_total`` vector on
    every rank and this rank's gradient slice (canonical layout of the shard)."""
    if dssim:
        vals, grad = dssim_with_gradient_(ssims_shard, grad_shard, imgs1_shard, imgs2_shard, None, True,
                                          divide_by_two_in_dssim)
    else:
        vals, grad = ssim_with_gradient_(ssims_shard, grad_shard, imgs1_shard, imgs2_shard, None, True)
    return gather_scores(vals, n_total, group), grad
