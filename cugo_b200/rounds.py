"""The running set of a batch of games, kept on the device from round to round.

A collector plays a batch of games in decision rounds: observe the running games,
choose their actions, step them.  Here the set of running games lives in device
memory as a list of row positions and its length: step_compact (the step kernel
with a round's bookkeeping) writes the next round's list and length, and the next
round's kernels read the length from memory.  So the host can launch round after
round without knowing how many games are still running; it learns that the batch
has finished from copies of the length taken every few rounds into pinned memory
behind events, read only once their event has completed (or a few newer copies are
queued), so the device queue never drains while the host waits.

Per game (indexed by row position): decisions taken, player 0's final reward, the
nagari flag; per batch: the count of bad step statuses.
"""
from __future__ import annotations

from typing import Any

import torch
from torch import nn


DONE_BYTE = 239  # TorchEnv50::done (a deal can end a game before its first decision)


class RunningSet:
    """The running games of `states` (rows [0, g)): the rows where `running` (bool
    [g], on the device; default: the rows whose done byte is 0, i.e. not ended at
    the deal) is set, in row order.  Built on the device without a host read: a
    stable sort puts the running rows first and their number is the count."""

    def __init__(self, ext, states: torch.Tensor, running: torch.Tensor | None = None,
                 check_every: int = 4, lookahead: int = 2, grouped: bool = False) -> None:
        dev = states.device
        g = states.shape[0]
        self.ext, self.states, self.g = ext, states, g
        i64 = dict(dtype=torch.int64, device=dev)
        # grouped: each round's list is grouped by the games' next decision (primary
        # plays, floor choices, prompts) instead of kept in row order, so a warp of
        # the next round runs one branch of the rule code (1.3-1.7x faster steps).
        self.grouped = grouped
        self.scratch = torch.empty(max(1, (6 if grouped else 2) * ((g + 31) // 32)),
                                   dtype=torch.int32, device=dev)
        self.counts = torch.empty(2, dtype=torch.int32, device=dev)
        self.bad = torch.empty(1, **i64)
        if running is None and dev.type == "cuda":
            # The games the deal did not end, in row order, and the zeroed per-game
            # arrays: three kernels (ext.running_init) instead of a sort and fills.  Every
            # entry of both id lists is a valid row (entries past the count are read).
            self.ids = (torch.empty(g, **i64), torch.empty(g, **i64))
            self.decision = torch.empty(g, dtype=torch.int32, device=dev)
            self.reward0 = torch.empty(g, dtype=torch.float32, device=dev)
            self.nagari = torch.empty(g, dtype=torch.bool, device=dev)
            ext.running_init(states, self.ids[0], self.counts[0:1], self.decision, self.reward0,
                             self.nagari, self.bad, self.scratch, spare_ids=self.ids[1])
        else:
            if running is None:
                running = states[:, DONE_BYTE] == 0
            # Running rows first, in order; the rest stay valid rows (read, not used).
            head = torch.sort((~running).to(torch.uint8), stable=True).indices
            self.ids = (head, torch.zeros(g, **i64))
            self.counts.zero_()
            self.counts[0:1].copy_(running.sum().view(1))
            self.decision = torch.zeros(g, dtype=torch.int32, device=dev)
            self.reward0 = torch.zeros(g, dtype=torch.float32, device=dev)
            self.nagari = torch.zeros(g, dtype=torch.bool, device=dev)
            self.bad.zero_()
        self._positions: torch.Tensor | None = None
        self.rounds = 0
        self.bound = g  # the host's upper bound of the running count
        self.check_every, self.lookahead = check_every, lookahead
        pin = dev.type == "cuda"
        self._seen = torch.zeros(lookahead + 1, dtype=torch.int32, pin_memory=pin)
        self._seen_extra = torch.zeros(lookahead + 1, dtype=torch.int64, pin_memory=pin)
        self.last_seen = (g, 0)
        self.last_seen_round = 0  # the round whose start the last copy read describes
        self._pending: list[tuple[torch.cuda.Event, int, int]] = []
        self._copies = 0
        self.done = g == 0

    @property
    def positions(self) -> torch.Tensor:
        """0 .. g - 1 (int64, made on first use)."""
        if self._positions is None:
            self._positions = torch.arange(self.g, dtype=torch.int64, device=self.states.device)
        return self._positions

    # -- the current round ---------------------------------------------------------
    @property
    def active(self) -> torch.Tensor:
        """Positions of the running games (entries past the count are stale)."""
        return self.ids[self.rounds & 1]

    @property
    def count(self) -> torch.Tensor:
        """The running count, int32 [1] in device memory."""
        k = self.rounds & 1
        return self.counts[k:k + 1]

    def step(self, actions: torch.Tensor, device_count: bool = True) -> None:
        """Steps the running games with actions[i] for position active[i] and moves to
        the next round.  device_count=False: the kernels step the first `bound` rows
        (the host's exact count, see read_count)."""
        k = self.rounds & 1
        active = self.ids[k] if device_count else self.ids[k][:self.bound]
        self.ext.step_compact(self.states, active, actions, self.decision, self.reward0,
                              self.nagari, self.bad, self.ids[1 - k], self.counts[1 - k:2 - k],
                              self.scratch, m_dev=self.counts[k:k + 1] if device_count else None,
                              grouped=self.grouped)
        self.rounds += 1

    def read_count(self) -> int:
        """The running count, read now (waits for the device)."""
        self.bound = int(self.count.item())
        self.done = self.bound == 0
        return self.bound

    def poll(self, extra: torch.Tensor | None = None) -> bool:
        """Every check_every rounds: queue a copy of the running count (and of
        `extra`, an int64 [1] device scalar) and look at the copies whose event has
        completed (waiting only when lookahead copies are queued).  Returns whether
        a copy showed no running game; the latest copy read is in last_seen (count,
        extra), taken when `last_seen_round` rounds had been stepped."""
        if self.done:
            return True
        if self.rounds % self.check_every:
            return False
        slot = self._copies % (self.lookahead + 1)
        self._copies += 1
        self._seen[slot:slot + 1].copy_(self.count, non_blocking=True)
        if extra is not None:
            self._seen_extra[slot:slot + 1].copy_(extra, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._pending.append((ev, slot, self.rounds))
        while self._pending and (len(self._pending) > self.lookahead or self._pending[0][0].query()):
            ev0, slot0, round0 = self._pending.pop(0)
            ev0.synchronize()
            self.last_seen = (int(self._seen[slot0]), int(self._seen_extra[slot0]))
            self.last_seen_round = round0
            self.bound = min(self.bound, self.last_seen[0])
            if self.last_seen[0] == 0:
                self.done = True
                break
        return self.done


def fused_sampler_params(model: nn.Module, features_width: int):
    """(bf16 weights, fp32 biases, activation code) of a model that the whole-network
    kernel runs with its sampling head, else None."""
    from .policy import ResidualMlpPolicy, fused_mlp_supported
    from .ppo import _ACT
    if isinstance(model, ResidualMlpPolicy):
        if model.samples_in_kernel() and model.inputs == features_width:
            return model.weights, model._fp32_biases(), _ACT[model.activation]
        return None
    weights = getattr(model, "_weights", None)
    if weights is None or getattr(model, "norm_kind", "none") != "none":
        return None
    ws, bs = weights([t for l in model.linears() for t in (l.weight, l.bias)])
    if (fused_mlp_supported(ws[0].shape[0], model.n_blocks, ws[0].shape[1], ws[-1].shape[0])
            and ws[-1].shape[0] >= 179 and ws[0].shape[1] == features_width):
        return ws, bs, _ACT[model.activation]
    return None


def choose_actions(ext: Any, model: nn.Module, fused, features, legal_bits, rows, seeds, decision,
            count, greedy: bool, seed_base: int):
    """Actions and log p of `model` on the running rows: the fused kernel reads the
    device count and each row's deal seed and decision count through `rows`; the
    generic path runs the forward and the sampler on the first `count` rows."""
    if fused is not None:
        ws, bs, act = fused
        actions, logp, _ = ext.mlp_fused_sample(features, ws, bs, act, legal_bits, seeds, decision,
                                                seed_base, greedy, m_dev=count, rows=rows)
        return actions, logp
    out = model(features)
    logits = (out[0] if isinstance(out, tuple) else out).float().contiguous()
    legal = unpack_legal(legal_bits)
    return ext.sample_actions(logits, legal, seeds.index_select(0, rows),
                              decision.index_select(0, rows), seed_base, greedy=greedy)


_BIT: dict = {}


def unpack_legal(bits: torch.Tensor) -> torch.Tensor:
    dev = bits.device
    if dev not in _BIT:
        a = torch.arange(179, device=dev)
        _BIT[dev] = (a // 64, a % 64)
    word, shift = _BIT[dev]
    return ((bits.index_select(1, word) >> shift) & 1).bool()
