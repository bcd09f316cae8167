"""GPU-resident self-play of the event-sequence policy in fixed-size waves.

The driver of the reference's WaveCollector (python/cugo_seq_selfplay50.py:36-238),
on the native engine and decode kernels: every tensor a decision step touches has
a fixed shape (finished games stay in the batch, masked), so one decision step —
observe, query token through the cached transformer, readout, Gumbel-max sample,
engine step, event record, event tokens for both seats into the KV cache — is
captured once as a CUDA graph and replayed; the wave reset (deal, opening tokens)
is a second graph.  The host replays graphs and checks every fourth step from the
16th whether the wave has finished (the reference's cadence).

Differences from the reference driver, by design of the benchmark: games are
dealt by the shared driver definition (game i: seed seed_base + i, first player
i & 1) and actions are sampled with the Philox Gumbel noise of
cugo_b200_sample_actions (counter {game, decision}) instead of torch.rand_like,
so runs are reproducible; the pool opponent of the reference (a frozen second
network for a subset of games) is not part of this driver.
"""
from __future__ import annotations

import torch

from .seq import MAX_EVENTS, QUERY_LD, SeqDecoder


class SeqWaveSelfPlay:
    def __init__(self, decoder: SeqDecoder, wave: int = 4096, max_steps: int = 64,
                 seed_base: int = 12345, record: bool = True, graphs: bool = True) -> None:
        self.dec, self.ext = decoder, decoder.ext
        dev = decoder.device
        self.w, self.max_steps, self.seed_base, self.record = wave, max_steps, seed_base, record
        w = wave
        i64 = dict(dtype=torch.int64, device=dev)
        self.ids = torch.arange(w, **i64)
        self.seats2 = torch.cat((torch.zeros(w, **i64), torch.ones(w, **i64)))
        self.game0 = torch.zeros(1, **i64)
        self.states = torch.zeros((w, self.ext.STATE_BYTES), dtype=torch.uint8, device=dev)
        self.events = torch.zeros((w, MAX_EVENTS, self.ext.EVENT_WORDS), **i64)
        self.count = torch.zeros(w, **i64)
        self.start = torch.zeros((w, self.ext.START_WORDS), **i64)
        self.decision = torch.zeros(w, dtype=torch.int32, device=dev)
        self.cache = decoder.new_cache(2 * w)  # row = seat * w + game
        self.query = torch.zeros((w, QUERY_LD), dtype=torch.bfloat16, device=dev)
        self.final_reward0 = torch.zeros(w, device=dev)
        self.final_nagari = torch.zeros(w, dtype=torch.bool, device=dev)
        self.finished = torch.zeros(w, dtype=torch.bool, device=dev)
        self.started = torch.zeros(w, dtype=torch.bool, device=dev)
        self.bad = torch.zeros((), **i64)
        self.step_index = torch.zeros(1, **i64)
        s = max_steps
        if record:  # what the trainer stores per decision (python/cugo_seq_selfplay50.py:68-75)
            self.rec_query = torch.zeros((s, w, QUERY_LD), dtype=torch.bfloat16, device=dev)
            self.rec_logp = torch.zeros((s, w), device=dev)
            self.rec_long = {k: torch.zeros((s, w), **i64) for k in ("actions", "seat", "count")}
            self.rec_valid = torch.zeros((s, w), dtype=torch.bool, device=dev)
        self.graphs = graphs
        self._reset_graph: torch.cuda.CUDAGraph | None = None
        self._step_graph: torch.cuda.CUDAGraph | None = None

    # -- the two captured bodies -------------------------------------------------
    def _reset(self) -> None:
        ext, dec, w = self.ext, self.dec, self.w
        games = self.game0 + self.ids
        self.states.copy_(ext.create(self.seed_base + games, games & 1))
        self.start.copy_(ext.start(self.states))
        self.events.zero_()
        self.count.zero_()
        self.decision.zero_()
        done = ext.observe_query_bf16(self.states, self.ids, query=self.query)[3]
        self.started.copy_(~done)
        self.finished.copy_(done)
        self.final_reward0.zero_()
        self.final_nagari.zero_()
        self.bad.zero_()
        self.step_index.zero_()
        if self.record:
            self.rec_valid.zero_()
        self.cache.length.zero_()
        x = dec.start_token(self.start, self.seats2)
        dec.cached_step(self.cache, x, slots=1)
        self.cache.length.fill_(1)

    def _step(self) -> None:
        ext, dec, w, ids = self.ext, self.dec, self.w, self.ids
        query, legal, players, done, status = ext.observe_query_bf16(self.states, ids, query=self.query)
        active = ~done
        self.bad += (active & ((status != 0) | ~legal.any(1))).sum()
        player = players.long()
        # One query per game on the mover's cache row.
        x = dec.query_token(query)
        dec.cached_step(self.cache, x, rows=(player & 1) * w + ids)
        logits = dec.readout(x)
        actions, logp = ext.sample_actions(logits, legal, self.game0 + ids, self.decision,
                                           seed_base=self.seed_base)
        if self.record:
            at = self.step_index
            self.rec_query.index_copy_(0, at, query.unsqueeze(0))
            self.rec_logp.index_copy_(0, at, logp.unsqueeze(0))
            for name, value in (("actions", actions), ("seat", player), ("count", self.count)):
                self.rec_long[name].index_copy_(0, at, value.unsqueeze(0))
            self.rec_valid.index_copy_(0, at, active.unsqueeze(0))
        reward0, new_done, nagari, step_status, committed, events = ext.step_events_indexed(
            self.states, ids, actions)
        self.bad += (active & (step_status != 0)).sum()
        finished_now = active & new_done
        self.final_reward0.copy_(torch.where(finished_now, reward0, self.final_reward0))
        self.final_nagari |= finished_now & nagari
        self.finished |= finished_now
        commit = active & committed
        slot = self.count.clamp_max(MAX_EVENTS - 1)
        self.events[ids, slot] = torch.where(commit.unsqueeze(1), events, self.events[ids, slot])
        # The event's token for both seats (row i of 2w reads event i % w).
        x2 = dec.event_token(events, self.seats2, self.count)
        dec.cached_step(self.cache, x2)
        self.cache.length += commit.repeat(2).long()
        self.count += commit.long()
        self.decision += active.int()
        self.step_index += 1

    def _capture(self) -> None:
        if self._step_graph is not None:
            return
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):  # warm-up outside the capture
                self._reset()
                self._step()
        torch.cuda.current_stream().wait_stream(side)
        self._reset_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._reset_graph):
            self._reset()
        self._step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._step_graph):
            self._step()

    # -- one wave ----------------------------------------------------------------
    def play_wave(self, game0: int) -> int:
        """Plays games game0 .. game0 + wave - 1 to the end; returns the steps taken."""
        self.game0.fill_(game0)
        if self.graphs:
            self._capture()
            self.game0.fill_(game0)
            self._reset_graph.replay()
        else:
            self._reset()
        steps = self.max_steps
        for k in range(self.max_steps):
            if self.graphs:
                self._step_graph.replay()
            else:
                self._step()
            if (k + 1) % 4 == 0 and k + 1 >= 16 and bool(self.finished.all()):
                steps = k + 1
                break
        else:
            if not bool(self.finished.all()):
                raise RuntimeError(f"games did not finish within {self.max_steps} steps")
        if int(self.bad):
            raise RuntimeError(f"{int(self.bad)} bad observe/step results in a wave")
        if int(self.count.max()) > MAX_EVENTS:
            raise RuntimeError("event log overflow")
        return steps

    def release(self) -> None:
        self._reset_graph = None
        self._step_graph = None
