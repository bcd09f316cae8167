"""Batched self-play: the decision loop of the reference's collect()
(python/cugo_ppo50.py:321-450) on this package's kernels.

Each decision round observes the live games, runs the policy, samples an action
per game with the Philox-addressed Gumbel-max kernel and steps the games; the live
set is compacted after every round.  The reference reads the live count back after
every round; with the fused policy step the kernels read it from device memory and
the host only polls copies of it (see play_batch).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .rounds import RunningSet


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


CHECK_EVERY = 4  # rounds between host reads of the running count (device-count loop)


def _log_actions(log: torch.Tensor, active: torch.Tensor, count: torch.Tensor,
                 decision: torch.Tensor, actions: torch.Tensor) -> None:
    """log[game, decision] = action for the first `count` running positions (count is
    a device tensor: no host read).  Positions past it write a spare last element."""
    flat = log.view(-1)
    width = log.shape[1]
    valid = torch.arange(active.numel(), device=active.device) < count
    d = decision.index_select(0, active).long()
    at = torch.where(valid & (d < width), active * width + d, flat.numel() - 1)
    flat.index_put_((at,), actions[:active.numel()].to(flat.dtype))


def play_batch(ext, policy, game_index: torch.Tensor, seed_base: int = 12345,
               max_rounds: int = 128, timer: RoundTimer | None = None,
               launches: list[int] | None = None,
               actions_log: torch.Tensor | None = None) -> BatchResult:
    """Plays games `game_index` (seed = seed_base + index, first player index & 1) to
    the end with policy-sampled actions.  A game that its deal already ended takes no
    decision and keeps reward 0 (as the reference's drivers count it).

    The running games are a device-resident list (rounds.RunningSet).  With a fused
    policy step (policy.samples_in_kernel()) the rounds run without host round trips:
    each round's kernels read the running count that the previous round's step left
    in device memory; every CHECK_EVERY rounds the host queues a copy of it and
    looks at copies whose event has completed, so the device never waits for the
    host.  Rounds launched after the count reached zero see zero rows and change
    nothing.  Otherwise (or with a timer, which needs each round's rows) the host
    reads the count after every round and sizes the next round's launches by it.

    actions_log (optional, for checking): int64 [games + 1, width]; entry [i, d]
    receives the action game i chose at its decision d (the extra last row takes the
    writes of positions past the running count)."""
    g = game_index.numel()
    states = ext.create_indexed(game_index, seed_base)  # seed_base + i, first player i & 1
    run = RunningSet(ext, states, check_every=CHECK_EVERY, grouped=True)
    fused = getattr(policy, "samples_in_kernel", lambda: False)()
    # The policy timer needs each round's row count: it reads the count every round.
    device_count = fused and timer is None
    # observe, the policy step, and step_compact's step, scan and scatter kernels
    per_round = 4 + getattr(policy, "launches_per_step", lambda: 1)()
    n_launch = 1
    while not run.done and run.rounds < max_rounds:
        if not device_count and run.read_count() == 0:
            break
        active, count = run.active, run.count
        if device_count:  # observe with bit-word masks, one policy kernel: no host reads
            features, legal, _p, _d, _s = ext.observe_indexed_bf16_bits(states, active, m_dev=count)
            t0 = timer.start() if timer else None
            # The kernel reads each row's game index and decision counter through active.
            actions, _logp = policy.forward_sample(features, legal, game_index, run.decision,
                                                   seed_base, m_dev=count, rows=active)
        else:
            active = active[:run.bound]
            features, legal, _p, _d, _s = (ext.observe_indexed_bf16_bits(states, active) if fused
                                           else ext.observe_indexed_bf16(states, active))
            game_ids = game_index.index_select(0, active)
            dec = run.decision.index_select(0, active)
            t0 = timer.start() if timer else None
            if hasattr(policy, "forward_sample"):
                actions, _logp = policy.forward_sample(features, legal, game_ids, dec, seed_base)
            else:
                actions, _logp = ext.sample_actions(policy(features), legal, game_ids, dec,
                                                    seed_base)
        if timer:
            timer.stop(t0, run.bound)
        if actions_log is not None:
            _log_actions(actions_log, active, count, run.decision, actions)
        run.step(actions, device_count)
        n_launch += per_round
        if device_count:
            run.poll()
    if not run.done and run.read_count() != 0:
        raise RuntimeError(f"games did not finish within {max_rounds} rounds")
    if launches is not None:
        launches.append(n_launch)
    if g == 0:
        return BatchResult(0, 0, 0, int(run.bad.item()), run.reward0, run.nagari)
    # One host read for the totals; every live game decides once per round, so the
    # most decisions of a game is the number of rounds played.
    decisions, played, bad = torch.stack([run.decision.sum(), run.decision.max().long(),
                                          run.bad[0]]).tolist()
    return BatchResult(g, decisions, played, bad, run.reward0, run.nagari)
