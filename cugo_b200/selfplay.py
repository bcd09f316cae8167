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
LOOKAHEAD = 2    # reads in flight: the host waits on a read only this many checks later


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
    the end with policy-sampled actions.

    With a fused policy step (policy.samples_in_kernel()) the rounds run without host
    round trips: each round's kernels read the running count that the previous
    round's step left in device memory (buffers keep the batch's full size).  Every
    CHECK_EVERY rounds the count is copied to pinned host memory behind an event; the
    host looks at a copy only once its event has completed (or LOOKAHEAD later
    copies are queued), so the device never waits for the host.  Rounds launched
    after the count reached zero see zero rows and change nothing.  Otherwise the
    host reads the count after every round and sizes the next round's launches by
    it.

    actions_log (optional, for checking): int64 [games + 1, width]; entry [i, d]
    receives the action game i chose at its decision d (the extra last row takes the
    writes of positions past the running count)."""
    device = game_index.device
    g = game_index.numel()
    states = ext.create(game_index + seed_base, game_index & 1)
    decision = torch.zeros(g, dtype=torch.int32, device=device)
    reward0 = torch.zeros(g, dtype=torch.float32, device=device)
    nagari = torch.zeros(g, dtype=torch.bool, device=device)
    bad = torch.zeros(1, dtype=torch.int64, device=device)
    # The running games' positions, written by the step kernel (ping-pong), their counts.
    # Entries past the count stay valid positions (they are gathered, not used).
    ids_buf = (torch.arange(g, device=device), torch.zeros(g, dtype=torch.int64, device=device))
    counts = torch.tensor([g, 0], dtype=torch.int32, device=device)
    scratch = torch.empty(2 * ((g + 31) // 32), dtype=torch.int32, device=device)
    fused = getattr(policy, "samples_in_kernel", lambda: False)()
    # The policy timer needs each round's row count: it reads the count every round.
    sync_each = not fused or timer is not None
    # observe, the policy step, and step_compact's step, scan and scatter kernels
    per_round = 4 + getattr(policy, "launches_per_step", lambda: 1)()
    n_launch = 1
    rounds = 0
    live = g
    # Copies of the running count in flight: (event, pinned slot).
    seen = torch.empty(LOOKAHEAD + 1, dtype=torch.int32, pin_memory=device.type == "cuda")
    pending: list[tuple[torch.cuda.Event, int]] = []
    n_copies = 0
    finished = False
    for rounds in range(1, max_rounds + 1):
        k = (rounds - 1) & 1
        active, nxt = ids_buf[k], ids_buf[1 - k]
        c_in, c_out = counts[k:k + 1], counts[1 - k:2 - k]
        if not fused:
            active = active[:live]
        if fused:  # observe with bit-word masks, one policy kernel, step: no host reads
            features, legal, _p, _d, _s = ext.observe_indexed_bf16_bits(states, active, m_dev=c_in)
            t0 = timer.start() if timer else None
            # The kernel reads each row's game index and decision counter through active.
            actions, _logp = policy.forward_sample(features, legal, game_index, decision, seed_base,
                                                   m_dev=c_in, rows=active)
        else:
            features, legal, _p, _d, _s = ext.observe_indexed_bf16(states, active)
            game_ids, dec = game_index.index_select(0, active), decision.index_select(0, active)
            t0 = timer.start() if timer else None
            if hasattr(policy, "forward_sample"):
                actions, _logp = policy.forward_sample(features, legal, game_ids, dec, seed_base)
            else:
                actions, _logp = ext.sample_actions(policy(features), legal, game_ids, dec,
                                                    seed_base)
        if timer:
            timer.stop(t0, live)
        if actions_log is not None:
            _log_actions(actions_log, active, c_in if fused else torch.tensor(live, device=device),
                         decision, actions)
        ext.step_compact(states, active, actions, decision, reward0, nagari, bad, nxt, c_out,
                         scratch, m_dev=c_in if fused else None)
        n_launch += per_round
        if sync_each:
            live = int(c_out.item())
            if live == 0:
                break
        elif rounds % CHECK_EVERY == 0:
            slot = n_copies % (LOOKAHEAD + 1)
            n_copies += 1
            seen[slot:slot + 1].copy_(c_out, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            pending.append((ev, slot))
            while pending and (len(pending) > LOOKAHEAD or pending[0][0].query()):
                ev0, slot0 = pending.pop(0)
                ev0.synchronize()
                if int(seen[slot0]) == 0:
                    finished = True
                    break
            if finished:
                break
    else:
        # The last round's count says whether the games ended within the limit.
        if max_rounds == 0 or int(c_out.item()) != 0:
            raise RuntimeError(f"games did not finish within {max_rounds} rounds")
    if launches is not None:
        launches.append(n_launch)
    decisions = int(decision.sum())
    played = int(decision.max()) if g else 0  # every live game decides once per round
    return BatchResult(g, decisions, played, int(bad), reward0, nagari)
