"""GPU-resident self-play of the event-sequence policy in fixed-size waves, the
driver behind the reference's WaveCollector (python/cugo_seq_selfplay50.py:36-238),
on the native engine and decode kernels.

A wave is `wave` games played together in fixed-shape buffers (finished games stay
in the batch and are skipped by the kernels' bookkeeping).  Two CUDA graphs:

  reset  deal the wave's games, their opening records and opening tokens (both
         seats' caches; the pool opponent's cache for pool games), zero the logs
  step   observe every game into the query rows; one pass of the cached
         transformer over the tokens the previous step left (its event's tokens for
         both seats' caches; at a wave's first step the opening tokens) and the query
         tokens on the mover's cache row, and the readout (and, in pool games where
         the opponent moves, the same for the opponent network on its own cache);
         Gumbel-max sampling; the engine step with its event words; the event's
         tokens embedded for the next step's pass; then one wave-tail kernel does the
         rest of the step's bookkeeping on the device: bad-status counts, final
         rewards, the event log, the per-decision records, the cache lengths, event
         counts and decision counters, and the wave's running count

One pass per step: the event tokens of step s and the query tokens of step s + 1
share every layer's LayerNorm and GEMM launches (rows 0 .. 2w - 1 and 2w .. 3w - 1
of one residual stream), with the events' attention (and cache append) before the
queries' at every layer -- the same arithmetic per row as an event pass followed by
a query pass, at half the launches.  The events of a wave's last step are never
embedded into the cache: no query follows them.

The host replays the step graph and, every 4 steps, copies the running count into
pinned memory behind an event and reads it; the wave ends at the first copy that
shows no running game (at most 3 steps after its last game ended; such steps change
nothing).

Sampling uses the Philox Gumbel noise of cugo_b200_sample_actions (counter {game,
decision}) instead of torch.rand_like, so a wave is reproducible.  Games are dealt
by the shared driver definition (game i: seed seed_base + i, first player i & 1).
Pool games are the first `pool_games` of each wave; there the learner plays seat
(i >> 1) & 1 of game i and the frozen opponent the other seat, and only the
learner's decisions are marked valid in the records.
"""
from __future__ import annotations

import torch

from .seq import MAX_EVENTS, QUERY_LD, SeqDecoder

POLL_EVERY = 4
# Copies of the running count the host lets run ahead of its reads.  A wave's steps
# have a fixed shape, so every step queued past the end costs a full step: the host
# reads each copy before queueing more (a short drain every POLL_EVERY steps).
LOOKAHEAD = 0


class SeqWaveSelfPlay:
    def __init__(self, decoder: SeqDecoder, wave: int = 4096, max_steps: int = 64,
                 seed_base: int = 12345, record: bool = True, graphs: bool = True,
                 opponent: SeqDecoder | None = None, pool_games: int = 0) -> None:
        self.dec, self.ext = decoder, decoder.ext
        self.opponent = opponent
        self.pool = min(pool_games, wave) if opponent is not None else 0
        dev = decoder.device
        self.w, self.max_steps, self.seed_base, self.record = wave, max_steps, seed_base, record
        w = wave
        i64 = dict(dtype=torch.int64, device=dev)
        self.ids = torch.arange(w, **i64)
        self.seats2 = torch.cat((torch.zeros(w, **i64), torch.ones(w, **i64)))
        self.game0 = torch.zeros(1, **i64)
        self.states = torch.zeros((w, self.ext.STATE_BYTES), dtype=torch.uint8, device=dev)
        self.start = torch.zeros((w, self.ext.START_WORDS), **i64)
        self.cache = decoder.new_cache(2 * w)  # row = seat * w + game
        self.query = torch.zeros((w, QUERY_LD), dtype=torch.bfloat16, device=dev)
        # The step's residual stream: the previous step's tokens for both seats' cache
        # rows, then the query rows; and the slots those tokens go to.
        self.x = torch.zeros((3 * w, decoder.d_model), dtype=torch.float32, device=dev)
        self.prev_pos = torch.zeros(2 * w, **i64)
        self.live = torch.ones(3 * w, dtype=torch.bool, device=dev)  # rows that attend
        self.started = torch.zeros(w, dtype=torch.bool, device=dev)
        # Device state the wave-tail kernel updates.
        self.state = {
            "final_reward0": torch.zeros(w, device=dev),
            "final_nagari": torch.zeros(w, dtype=torch.bool, device=dev),
            "finished": torch.zeros(w, dtype=torch.bool, device=dev),
            "bad": torch.zeros(1, **i64),
            "running": torch.zeros(1, dtype=torch.int32, device=dev),
            "events": torch.zeros((w, MAX_EVENTS, self.ext.EVENT_WORDS), **i64),
            "count": torch.zeros(w, **i64),
            "cache_length": self.cache.length,
            "decision": torch.zeros(w, dtype=torch.int32, device=dev),
            "step_index": torch.zeros(1, **i64),
        }
        self.records = None
        if record:  # what the trainer stores per decision (python/cugo_seq_selfplay50.py:68-75)
            s = max_steps
            self.rec_query = torch.zeros((s, w, QUERY_LD), dtype=torch.bfloat16, device=dev)
            self.records = {"actions": torch.zeros((s, w), **i64), "seat": torch.zeros((s, w), **i64),
                            "count": torch.zeros((s, w), **i64),
                            "logp": torch.zeros((s, w), device=dev),
                            "valid": torch.zeros((s, w), dtype=torch.bool, device=dev)}
        if self.pool:
            p = self.pool
            self.opp_cache = opponent.new_cache(p)  # row = pool game (the opponent's seat)
            self.opp_x = torch.zeros((2 * p, opponent.d_model), dtype=torch.float32, device=dev)
            self.opp_prev_pos = torch.zeros(p, **i64)
            self.learner_seat = (self.ids[:p] >> 1) & 1
            self.opp_seat = 1 - self.learner_seat
            self.learner = torch.ones(w, dtype=torch.bool, device=dev)
        self.graphs = graphs
        self._reset_graph: torch.cuda.CUDAGraph | None = None
        self._step_graph: torch.cuda.CUDAGraph | None = None
        pin = dev.type == "cuda"
        self._seen = torch.zeros(LOOKAHEAD + 1, dtype=torch.int32, pin_memory=pin)

    # -- readable views of the wave's device state -----------------------------------
    @property
    def events(self) -> torch.Tensor:
        return self.state["events"]

    @property
    def count(self) -> torch.Tensor:
        return self.state["count"]

    @property
    def final_reward0(self) -> torch.Tensor:
        return self.state["final_reward0"]

    @property
    def final_nagari(self) -> torch.Tensor:
        return self.state["final_nagari"]

    @property
    def finished(self) -> torch.Tensor:
        return self.state["finished"]

    @property
    def decision(self) -> torch.Tensor:
        return self.state["decision"]

    # -- the two captured bodies -------------------------------------------------------
    def _reset(self) -> None:
        ext, dec, st = self.ext, self.dec, self.state
        games = self.game0 + self.ids
        self.states.copy_(ext.create(self.seed_base + games, games & 1))
        self.start.copy_(ext.start(self.states))
        for name in ("events", "count", "decision", "final_reward0", "final_nagari", "bad",
                     "step_index"):
            st[name].zero_()
        done = ext.observe_query_bf16(self.states, self.ids, query=self.query)[3]
        self.started.copy_(~done)
        st["finished"].copy_(done)
        st["running"].copy_(self.started.sum())
        if self.records is not None:
            self.records["valid"].zero_()
        # The opening tokens go to slot 0 in the first step's pass.
        dec.start_token(self.start, self.seats2, out=self.x[:2 * self.w])
        self.prev_pos.zero_()
        self.cache.length.fill_(1)
        if self.pool:
            p = self.pool
            opp = self.opponent
            opp.start_token(self.start[:p], self.opp_seat, out=self.opp_x[:p])
            self.opp_prev_pos.zero_()
            self.opp_cache.length.fill_(1)

    def _step(self) -> None:
        ext, dec, w, ids, st = self.ext, self.dec, self.w, self.ids, self.state
        query, legal, players, done, status = ext.observe_query_bf16(self.states, ids, query=self.query)
        seat = players.long() & 1
        x = dec.query_token(query, out=self.x[2 * w:])
        # Games that finished before this step feed no later decision: their tokens
        # neither attend nor append (the wave tail leaves their records alone).
        live = ~done
        self.live.copy_(torch.cat((live, live, live)))
        dec.cached_step_segments(self.cache, self.x, [(2 * w, None, self.prev_pos),
                                                      (w, seat * w + ids, self.cache.length)],
                                 active=self.live)
        logits = dec.readout(x)
        if self.pool:
            p, opp = self.pool, self.opponent
            xo = opp.query_token(query[:p], out=self.opp_x[p:])
            opp.cached_step_segments(self.opp_cache, self.opp_x,
                                     [(p, None, self.opp_prev_pos), (p, None, self.opp_cache.length)],
                                     active=torch.cat((live[:p], live[:p])))
            theirs = seat[:p] != self.learner_seat
            logits[:p] = torch.where(theirs.unsqueeze(1), opp.readout(xo)[:, :logits.shape[1]],
                                     logits[:p])
            self.learner[:p] = ~theirs
        actions, logp = ext.sample_actions(logits, legal, self.game0 + ids, st["decision"],
                                           seed_base=self.seed_base)
        if self.records is not None:
            self.rec_query.index_copy_(0, st["step_index"].clamp_max(self.max_steps - 1),
                                       query.unsqueeze(0))
        step_out = ext.step_events_indexed(self.states, ids, actions)
        events = step_out[5]
        # The event's tokens for both seats (row i of 2w reads event i % w), at the
        # games' event counts before this step, for the next step's pass at the slots
        # the cache lengths give now (the wave tail advances them).
        self.prev_pos.copy_(self.cache.length)
        dec.event_token(events, self.seats2, st["count"], out=self.x[:2 * w])
        if self.pool:
            p, opp = self.pool, self.opponent
            self.opp_prev_pos.copy_(self.opp_cache.length)
            opp.event_token(events[:p], self.opp_seat, st["count"][:p], out=self.opp_x[:p])
            self.opp_cache.length += (step_out[4][:p] & ~done[:p]).long()
        ext.wave_tail(done, status, players, actions, logp, step_out, st, self.records,
                      learner=self.learner if self.pool else None)

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

    # -- one wave ------------------------------------------------------------------------
    def play_wave(self, game0: int) -> int:
        """Plays games game0 .. game0 + wave - 1 to the end; returns the steps run."""
        self.game0.fill_(game0)
        if self.graphs:
            self._capture()
            self.game0.fill_(game0)
            self._reset_graph.replay()
        else:
            self._reset()
        pending: list[tuple[torch.cuda.Event, int, int]] = []
        copies, steps, ended = 0, 0, None
        for k in range(1, self.max_steps + 1):
            self._step_graph.replay() if self.graphs else self._step()
            steps = k
            if k % POLL_EVERY:
                continue
            slot = copies % (LOOKAHEAD + 1)
            copies += 1
            self._seen[slot:slot + 1].copy_(self.state["running"], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            pending.append((ev, slot, k))
            while pending and (len(pending) > LOOKAHEAD or pending[0][0].query()):
                ev0, slot0, at = pending.pop(0)
                ev0.synchronize()
                if int(self._seen[slot0]) == 0:
                    ended = at
                    break
            if ended is not None:
                break
        torch.cuda.synchronize()
        st = self.state
        running, bad, longest = (int(v) for v in torch.stack(
            (st["running"][0].long(), st["bad"][0], st["count"].max())).tolist())
        if running:
            raise RuntimeError(f"games did not finish within {self.max_steps} steps")
        if bad:
            raise RuntimeError(f"{bad} bad observe/step results in a wave")
        if longest > MAX_EVENTS:
            raise RuntimeError("event log overflow")
        return ended if ended is not None else steps

    def release(self) -> None:
        self._reset_graph = None
        self._step_graph = None
