"""Batched self-play: the decision loop of the reference's collect()
(python/cugo_ppo50.py:321-450) on this package's kernels.

Each decision round observes the live games, runs the policy, samples an action
per game with the Philox-addressed Gumbel-max kernel and steps the games; the live
set is compacted after every round (one device->host read of its size, as the
reference's compaction does).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class BatchResult:
    games: int
    decisions: int
    rounds: int
    bad_status: int
    reward0: torch.Tensor  # fp32 [games], player 0's final reward
    nagari: torch.Tensor   # bool [games]


@dataclass
class RoundTimer:
    """Optional CUDA-event bracketing of the policy forward inside each round."""
    enabled: bool = False

    def __post_init__(self) -> None:
        self.pairs: list[tuple[torch.cuda.Event, torch.cuda.Event, int]] = []

    def start(self):
        if not self.enabled:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def stop(self, start, rows: int) -> None:
        if start is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.pairs.append((start, e, rows))

    def total_ms(self) -> tuple[float, int, int]:
        ms = sum(a.elapsed_time(b) for a, b, _ in self.pairs)
        return ms, len(self.pairs), sum(r for _, _, r in self.pairs)


def play_batch(ext, policy, game_index: torch.Tensor, seed_base: int = 12345,
               max_rounds: int = 128, timer: RoundTimer | None = None,
               launches: list[int] | None = None) -> BatchResult:
    """Plays games `game_index` (seed = seed_base + index, first player index & 1) to
    the end with policy-sampled actions."""
    device = game_index.device
    g = game_index.numel()
    states = ext.create(game_index + seed_base, game_index & 1)
    decision = torch.zeros(g, dtype=torch.int32, device=device)
    reward0 = torch.zeros(g, dtype=torch.float32, device=device)
    nagari = torch.zeros(g, dtype=torch.bool, device=device)
    bad = torch.zeros((), dtype=torch.int64, device=device)
    active = torch.arange(g, device=device)
    decisions = 0
    rounds = 0
    n_launch = 1
    for rounds in range(1, max_rounds + 1):
        fused = getattr(policy, "samples_in_kernel", lambda: False)()
        # A fused policy step reads the legal mask as bit words.
        observe = ext.observe_indexed_bf16_bits if fused else ext.observe_indexed_bf16
        features, legal, _players, _done, status = observe(states, active)
        game_ids = game_index.index_select(0, active)
        dec = decision.index_select(0, active)
        t0 = timer.start() if timer else None
        if hasattr(policy, "forward_sample"):  # policy and sampling in one launch where fused
            actions, _logp = policy.forward_sample(features, legal, game_ids, dec, seed_base)
        else:
            actions, _logp = ext.sample_actions(policy(features), legal, game_ids, dec, seed_base)
        if timer:
            timer.stop(t0, active.numel())
        reward, new_done, new_nagari, step_status, _ = ext.step_indexed(states, active, actions)
        n_launch += 2 + getattr(policy, "launches_per_step", lambda: 1)()
        bad += ((step_status != 0) & (step_status != 9)).sum()
        decisions += active.numel()
        decision.index_add_(0, active, torch.ones_like(active, dtype=torch.int32))
        reward0.index_copy_(0, active, torch.where(new_done, reward, 0.0))
        nagari.index_copy_(0, active, new_done & new_nagari)
        active = active.index_select(0, torch.nonzero(~new_done).squeeze(1))
        if active.numel() == 0:
            break
    else:
        raise RuntimeError(f"games did not finish within {max_rounds} rounds")
    if launches is not None:
        launches.append(n_launch)
    return BatchResult(g, decisions, rounds, int(bad), reward0, nagari)
