"""Batch sharding over the GPUs of one node (one process per GPU).

Images are independent (the reference loops over them, src/core.jl:186), so a
batch splits into contiguous slices with no exchange in the data path.  The
only communication is one all-gather of the per-image (D)SSIM scalars, so every
rank ends with the full vector while each rank's gradient slice stays resident
on its own GPU.  With the NCCL backend the all-gather runs over NVLink.
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from .interface import dssim_with_gradient_, ssim_with_gradient_


class CollectiveTimeout(RuntimeError):
    """A collective did not complete within its host deadline: a peer rank died,
    hangs, or never joined.  Call ``abort_group`` before leaving, so that no rank
    stays blocked in the communicator."""


def _wait(work, deadline_s: float | None, what: str) -> None:
    """Wait for an async collective, polling its completion against a host deadline.

    With NCCL, ``is_completed`` queries the collective's CUDA event, so polling
    also waits for the kernels queued before it on the stream."""
    if deadline_s is None:
        work.wait()
        return
    t_end = time.monotonic() + deadline_s
    while not work.is_completed():
        if time.monotonic() > t_end:
            raise CollectiveTimeout(f"{what}: not completed within {deadline_s:g} s on rank "
                                    f"{dist.get_rank()} of {dist.get_world_size()}")
        time.sleep(2e-4)
    work.wait()   # raises an error the backend recorded for the collective


def abort_group(group=None) -> None:
    """Abort the communicator of ``group`` after a ``CollectiveTimeout`` (ncclCommAbort
    for NCCL; gloo returns once the peers' connections close).  torch exposes the
    abort only through this internal hook."""
    dist.distributed_c10d._abort_process_group(group)


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of n images for `rank` (the first n % world ranks get one more)."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def gather_scores(local: torch.Tensor, n_total: int, group=None, deadline_s: float | None = None) -> torch.Tensor:
    """All-gather per-image scores of unequal shards into one length-n_total vector.

    With ``deadline_s`` the host polls the collective and raises ``CollectiveTimeout``
    once the deadline passes (a rank that died or never joined), instead of
    blocking until the process group's own timeout."""
    world = dist.get_world_size(group)
    per = -(-n_total // world)
    buf = torch.zeros(per, dtype=local.dtype, device=local.device)
    buf[: local.numel()].copy_(local)
    out = torch.empty(per * world, dtype=local.dtype, device=local.device)
    work = dist.all_gather_into_tensor(out, buf, group=group, async_op=True)
    _wait(work, deadline_s, "all-gather of per-image scores")
    parts = []
    for r in range(world):
        lo, hi = shard_range(n_total, world, r)
        parts.append(out[r * per: r * per + (hi - lo)])
    return torch.cat(parts)


class ScoreGather:
    """A reusable all-gather of per-image scores, for a loop that gathers every step.

    The padded send buffer and the output are allocated once.  When every shard has
    the same length, the shard is gathered straight into the output (no padding, no
    concatenation).  ``start`` issues the collective asynchronously and returns its
    handle; the caller may launch the next step's kernel before waiting on it, as long
    as that kernel does not overwrite the scores being sent (use two score buffers in
    turn).  ``finish`` waits (with the optional host deadline of ``gather_scores``) and
    returns the full length-``n_total`` vector."""

    def __init__(self, n_total: int, dtype, device, group=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.n_total = n_total
        self.per = -(-n_total // self.world)
        self.equal = self.per * self.world == n_total
        self.out = torch.empty(self.per * self.world, dtype=dtype, device=device)
        self.buf = None if self.equal else torch.zeros(self.per, dtype=dtype, device=device)
        if not self.equal:
            idx = []
            for r in range(self.world):
                lo, hi = shard_range(n_total, self.world, r)
                idx.extend(range(r * self.per, r * self.per + (hi - lo)))
            self.index = torch.tensor(idx, dtype=torch.long, device=device)

    def start(self, local: torch.Tensor):
        if self.equal:
            src = local
        else:
            self.buf[: local.numel()].copy_(local)
            src = self.buf
        return dist.all_gather_into_tensor(self.out, src, group=self.group, async_op=True)

    def finish(self, work, deadline_s: float | None = None) -> torch.Tensor:
        _wait(work, deadline_s, "all-gather of per-image scores")
        return self.out if self.equal else self.out.index_select(0, self.index)


def sharded_with_gradient(imgs1_shard, imgs2_shard, n_total: int, dssim: bool = False,
                          divide_by_two_in_dssim: bool = False, ssims_shard=None, grad_shard=None,
                          group=None, deadline_s: float | None = None):
    """(D)SSIM with gradient on this rank's shard, then the all-gather of the scores.

    Returns ``(all_scores, grad_shard)``: the full length-``n_total`` vector on
    every rank and this rank's gradient slice (canonical layout of the shard).
    ``deadline_s`` bounds the all-gather (see ``gather_scores``)."""
    if dssim:
        vals, grad = dssim_with_gradient_(ssims_shard, grad_shard, imgs1_shard, imgs2_shard, None, True,
                                          divide_by_two_in_dssim)
    else:
        vals, grad = ssim_with_gradient_(ssims_shard, grad_shard, imgs1_shard, imgs2_shard, None, True)
    return gather_scores(vals, n_total, group, deadline_s), grad
