"""Host-side plumbing of multi-GPU self-play: one process per GPU, games sharded by
disjoint seed blocks, only episode statistics (and timings) reduced across ranks.

Self-play has no data-path collective: rank r, step s plays the game block
[(s * world + r) * games, + games) (game i: seed 12345 + i, first player i & 1), so
the union over ranks and steps is a contiguous range and no game is played twice.
The reductions run over whatever process group is initialised (NCCL on the GPU
box, gloo in the CPU tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def block_start(step: int, rank: int, world: int, games: int) -> int:
    """First game index of rank `rank`'s block at step `step`."""
    return (step * world + rank) * games


def game_block(step: int, rank: int, world: int, games: int,
               device: torch.device | str = "cuda") -> torch.Tensor:
    """Game indices of one rank's block (int64 on `device`)."""
    return torch.arange(games, dtype=torch.int64, device=device) + block_start(step, rank, world, games)


def all_reduce(values: list[float], world: int, op: str = "sum",
               device: torch.device | str = "cuda") -> list[float]:
    """Sums (or maxima) of per-rank statistics, as float64."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX)
    return t.tolist()


def all_gather(values: list[float], world: int,
               device: torch.device | str = "cuda") -> list[list[float]]:
    """Every rank's list of statistics (float64), in rank order."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world == 1:
        return [t.tolist()]
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [p.tolist() for p in parts]
