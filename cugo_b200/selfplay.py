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
    bad = torch.zeros(1, dtype=torch.int64, device=device)
    active = torch.arange(g, device=device)
    # The games still running after a round, written by the step kernel (ping-pong).
    ids_buf = (torch.empty(g, dtype=torch.int64, device=device),
               torch.empty(g, dtype=torch.int64, device=device))
    count = torch.zeros(1, dtype=torch.int32, device=device)
    scratch = torch.empty(2 * ((g + 31) // 32), dtype=torch.int32, device=device)
    decisions = 0
    rounds = 0
    n_launch = 1
    fused = getattr(policy, "samples_in_kernel", lambda: False)()
    # A fused policy step reads the legal mask as bit words.
    observe = ext.observe_indexed_bf16_bits if fused else ext.observe_indexed_bf16
    for rounds in range(1, max_rounds + 1):
        features, legal, _players, _done, _status = observe(states, active)
        game_ids = game_index.index_select(0, active)
        dec = decision.index_select(0, active)
        t0 = timer.start() if timer else None
        if hasattr(policy, "forward_sample"):  # policy and sampling in one launch where fused
            actions, _logp = policy.forward_sample(features, legal, game_ids, dec, seed_base)
        else:
            actions, _logp = ext.sample_actions(policy(features), legal, game_ids, dec, seed_base)
        if timer:
            timer.stop(t0, active.numel())
        nxt = ids_buf[rounds & 1]
        ext.step_compact(states, active, actions, decision, reward0, nagari, bad, nxt, count, scratch)
        n_launch += 2 + getattr(policy, "launches_per_step", lambda: 1)()
        decisions += active.numel()
        live = int(count.item())  # the round's one device->host read
        if live == 0:
            break
        active = nxt[:live]
    else:
        raise RuntimeError(f"games did not finish within {max_rounds} rounds")
    if launches is not None:
        launches.append(n_launch)
    return BatchResult(g, decisions, rounds, int(bad), reward0, nagari)
