"""Multi-GPU host logic for the fused operators: one process per GPU, M (token rows) or
the conv batch split into contiguous shards, weights replicated.  The operators need no
communication; `gather_rows` concatenates the row shards on every rank (NCCL all-gather
over NVLink on GPUs, gloo on CPU) for callers that need the whole output on one device,
and `StepGuard` lets ranks notice a lost peer between steps, on the host, before any
kernel or collective of the next step is launched.
"""
from __future__ import annotations

import datetime
from typing import Optional, Tuple

import torch
import torch.distributed as dist


def row_shard(M: int, world: int, rank: int, align: int = 128) -> Tuple[int, int]:
    """[lo, hi) rows of `rank`: contiguous, in multiples of `align` rows (one 128-row tile)
    so no tile straddles two ranks; the last rank takes the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    blocks = -(-M // align)
    per, extra = divmod(blocks, world)
    lo_b = rank * per + min(rank, extra)
    hi_b = lo_b + per + (1 if rank < extra else 0)
    return min(M, lo_b * align), min(M, hi_b * align)


def gather_rows(shard: torch.Tensor, M: int, group=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Concatenate every rank's row shard (as produced by row_shard) into [M, ...] on
    every rank (into `out` when given).  Equal shards are gathered straight into the
    output with one all-gather; shards of different lengths are padded to the longest
    for the collective and trimmed after."""
    world = dist.get_world_size(group)
    sizes = [row_shard(M, world, r) for r in range(world)]
    longest = max(hi - lo for lo, hi in sizes)
    if all(hi - lo == longest for lo, hi in sizes) and shard.is_contiguous():
        if out is None:
            out = torch.empty((M,) + tuple(shard.shape[1:]), dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(out, shard, group=group)
        return out
    pad = torch.zeros((longest,) + tuple(shard.shape[1:]), dtype=shard.dtype, device=shard.device)
    pad[: shard.shape[0]] = shard
    buf = torch.empty((world * longest,) + tuple(shard.shape[1:]), dtype=shard.dtype, device=shard.device)
    dist.all_gather_into_tensor(buf, pad, group=group)
    rows = torch.cat([buf[r * longest: r * longest + (hi - lo)] for r, (lo, hi) in enumerate(sizes)])
    if out is not None:
        out.copy_(rows)
        return out
    return rows


class PeerLost(RuntimeError):
    """A rank did not check in for a step within the timeout."""


class StepGuard:
    """Host-side liveness check between steps through the process group's key-value
    store: every rank checks in for step k and waits (bounded) for all others before it
    launches step k's kernels.  A rank that raised, exited or hangs is reported as
    PeerLost instead of leaving the survivors blocked in a collective."""

    def __init__(self, store: dist.Store, world: int, rank: int, timeout_s: float = 30.0, prefix: str = "fo"):
        self.store, self.world, self.rank = store, world, rank
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix
        self.step = 0

    def check_in(self) -> None:
        k = self.step
        self.store.set(f"{self.prefix}/step{k}/rank{self.rank}", "1")
        keys = [f"{self.prefix}/step{k}/rank{r}" for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception as e:  # the store raises on timeout
            missing = [r for r in range(self.world) if not self.store.check([keys[r]])]
            raise PeerLost(f"step {k}: ranks {missing} did not check in within {self.timeout}") from e
        self.step += 1


def sharded_apply(fn, a: torch.Tensor, world: int, rank: int, align: int = 128) -> Tuple[torch.Tensor, int, int]:
    """Run fn on this rank's row shard of `a` (rows [lo, hi)); returns (out, lo, hi)."""
    lo, hi = row_shard(a.shape[0], world, rank, align)
    return fn(a[lo:hi]), lo, hi


__all__ = ["PeerLost", "StepGuard", "gather_rows", "row_shard", "sharded_apply"]
