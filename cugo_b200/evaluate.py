"""Paired evaluation of two policies on the native kernels: the reference's
evaluate_paired and league match (python/cugo_eval50.py:137-361,
python/league50.py:29-50), same arguments and summary.

Each deal is played twice with the seats swapped (games i and i + pairs share seed
i; policy A sits at seat 0 in the first half and seat 1 in the second).  The
reference compacts the running games on the host every decision step (three
nonzero() synchronisations per step, index copies for each policy's rows).  Here
every tensor keeps the full batch shape and one decision step is one CUDA graph:

  observe (bf16 features)  ->  rows sorted by who moves (A, then B, then finished)
  ->  policy A's layers on the window [0, nA), policy B's on [nA, nA + nB) of the
  sorted rows (the GEMM reads the window from device memory)  ->  masked argmax
  (or Gumbel-max sampling) in the sampler kernel  ->  actions scattered back  ->
  step  ->  running mask, final scores and failure counts updated on the device.

The host replays the graph and reads one flag every few steps.  Results equal the
reference loop's for the same policy forward (the tests compare both).  Sampling
draws Gumbel noise from Philox (counter {game, decision}, seed = seed_offset)
instead of torch.multinomial: the same distribution, reproducible.  Policies are
residual MLPs with norm "none" (PpoActor/FusedResidualMlp/ResidualMlpPolicy
layouts); sequence policies (uses_history) are not supported here.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Any

import torch

from .ext import load_extension

SIGNED_GOLDEN = -7046029254386353131  # python/cugo_ppo_nets50.py:11
SEED_BASE = 0x243F6A8885A308D3        # python/cugo_ppo_nets50.py:12
_ACT = {"relu": 1, "silu": 2}
CHECK_EVERY = 4  # decision steps between host reads of the running flag


def make_seeds(batch: int, offset: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Deal seeds and first players (python/cugo_ppo_nets50.py:15-17, int64 wrap)."""
    index = torch.arange(batch, dtype=torch.int64, device=device)
    return index.mul(SIGNED_GOLDEN).add(SEED_BASE + offset), index.bitwise_and(1)


def chunk_offset(seed_offset: int, start: int) -> int:
    """Seed offset whose first deal is deal `start` of a match at seed_offset
    (python/league50.py:25-28)."""
    seed = (SEED_BASE + seed_offset + start * SIGNED_GOLDEN + 2 ** 63) % 2 ** 64 - 2 ** 63
    return seed - SEED_BASE


@dataclass
class EvalSummary:
    """python/cugo_eval50.py:26-60."""
    pairs: int
    games: int
    evaluated_pairs: int
    evaluated_games: int
    predecision_excluded: int
    a_wins: int
    b_wins: int
    draws: int
    a_p0_wins: int
    a_p0_losses: int
    a_p0_draws: int
    a_p1_wins: int
    a_p1_losses: int
    a_p1_draws: int
    pair_wins: int
    pair_losses: int
    pair_draws: int
    mean_score_a: float
    mean_score_a_p0: float
    mean_score_a_p1: float
    mean_pair_score_a: float
    pair_score_std: float
    pair_score_se: float
    pair_score_ci95_low: float
    pair_score_ci95_high: float
    terminal: int
    nagari: int
    decision_steps: int
    seconds: float

    @property
    def games_per_s(self) -> float:
        return self.games / self.seconds


class WindowedMlp:
    """A residual-MLP policy (norm "none") run over a device-resident row window of
    fixed-capacity buffers: every layer is one window GEMM (bias, activation,
    residual in the epilogue), so the rows a policy plays can change between graph
    replays without a host round trip."""

    def __init__(self, ext: Any, model: Any, capacity: int, device: torch.device,
                 activation: str | None = None) -> None:
        self.ext = ext
        ws, bs, act = _mlp_params(model, activation)
        self.act = _ACT[act]
        self.w = [w.to(device, torch.bfloat16).contiguous() for w in ws]
        self.b = [b.to(device, torch.float32).contiguous() for b in bs]
        if self.w[0].shape[1] % 8:
            raise ValueError("the input width must be a multiple of 8")
        hidden = self.w[0].shape[0]
        self.blocks = (len(self.w) - 2) // 2
        self.outputs = self.w[-1].shape[0]
        self.h = torch.empty((capacity, hidden), dtype=torch.bfloat16, device=device)
        self.u = torch.empty((capacity, hidden), dtype=torch.bfloat16, device=device)

    def __call__(self, x: torch.Tensor, window: torch.Tensor, out: torch.Tensor) -> None:
        lin, w, b, act = self.ext.linear, self.w, self.b, self.act
        lin(x, w[0], b[0], out=self.h, act=act if self.blocks == 0 else 0, window=window)
        for i in range(self.blocks):
            lin(self.h, w[1 + 2 * i], b[1 + 2 * i], out=self.u, act=act, window=window)
            lin(self.u, w[2 + 2 * i], b[2 + 2 * i], residual=self.h, out=self.h,
                act_after=act if i == self.blocks - 1 else 0, window=window)
        lin(self.h, w[-1], b[-1], out=out, window=window)


def _mlp_params(model: Any, activation: str | None):
    """Weights, biases and activation of a ResidualMlp-layout policy: an nn.Module
    with inp / blocks.i.fc1 / blocks.i.fc2 / out (PpoActor, FusedResidualMlp), or a
    ResidualMlpPolicy."""
    if hasattr(model, "weights") and hasattr(model, "biases") and not hasattr(model, "state_dict"):
        return list(model.weights), list(model.biases), activation or model.activation
    state = model.state_dict()
    if any(".norm." in k or k.startswith("norm.") for k in state):
        raise ValueError("only norm 'none' residual MLPs run on the fused evaluator")
    blocks = len({k.split(".")[1] for k in state if k.startswith("blocks.")})
    names = ["inp"] + [f"blocks.{i}.fc{j}" for i in range(blocks) for j in (1, 2)] + ["out"]
    ws = [state[f"{n}.weight"].detach() for n in names]
    bs = [state[f"{n}.bias"].detach() for n in names]
    act = activation or getattr(model, "activation", "silu")
    if act not in _ACT:
        raise ValueError(f"activation {act!r}: relu or silu")
    return ws, bs, act


class PairedEvaluator:
    """The fixed-shape evaluation loop for `pairs` deal pairs (reused across calls of
    the same size, so its CUDA graph is captured once)."""

    def __init__(self, ext: Any, model_a: Any, model_b: Any, pairs: int,
                 device: torch.device | None = None, graphs: bool = True) -> None:
        self.ext = ext
        dev = self.device = device or torch.device("cuda")
        g = self.games = 2 * pairs
        self.pairs = pairs
        self.net_a = WindowedMlp(ext, model_a, g, dev)
        self.net_b = WindowedMlp(ext, model_b, g, dev)
        if self.net_a.outputs < ext.ACTION_COUNT or self.net_b.outputs < ext.ACTION_COUNT:
            raise ValueError("policies must output at least 179 logits")
        i64 = dict(dtype=torch.int64, device=dev)
        self.ids = torch.arange(g, **i64)
        self.a_seat = (self.ids >= pairs).to(torch.int64)
        self.states = torch.zeros((g, ext.STATE_BYTES), dtype=torch.uint8, device=dev)
        width = max(self.net_a.outputs, self.net_b.outputs)
        self.logits = torch.zeros((g, (width + 3) // 4 * 4), device=dev)
        self.win_a = torch.zeros(2, dtype=torch.int32, device=dev)
        self.win_b = torch.zeros(2, dtype=torch.int32, device=dev)
        self.running = torch.zeros(g, dtype=torch.bool, device=dev)
        self.final_reward0 = torch.zeros(g, device=dev)
        self.final_nagari = torch.zeros(g, dtype=torch.bool, device=dev)
        self.predecision_done = torch.zeros(g, dtype=torch.bool, device=dev)
        self.decision = torch.zeros(g, dtype=torch.int32, device=dev)
        self.bad = torch.zeros(3, **i64)  # observe, legal, step failures
        self.steps = torch.zeros((), **i64)
        self.sample = (False, False)
        self.graphs = graphs
        self._graph: torch.cuda.CUDAGraph | None = None
        self._graph_sample: tuple[bool, bool] | None = None
        self._graph_seed: int | None = None
        self._seed_value = 0

    # -- one decision step (captured) ------------------------------------------
    def _step(self) -> None:
        ext, g = self.ext, self.games
        features, legal, players, odone, status = ext.observe_indexed_bf16(self.states, self.ids)
        run = self.running
        ok = status == int(ext.STATUS_OK)
        has_legal = legal.any(1)
        self.bad[0] += (run & ~ok).sum()
        self.bad[1] += (run & ok & (odone | ~has_legal)).sum()
        use_a = run & (players.to(torch.int64) == self.a_seat)
        key = torch.where(use_a, 0, torch.where(run, 1, 2)).to(torch.int8)
        order = torch.sort(key, stable=True).indices
        n_a = use_a.sum().to(torch.int32)
        n_run = run.sum().to(torch.int32)
        self.win_a[1] = n_a
        self.win_b[0] = n_a
        self.win_b[1] = n_run - n_a
        feats = features.index_select(0, order)
        legal_s = legal.index_select(0, order)
        self.net_a(feats, self.win_a, self.logits)
        self.net_b(feats, self.win_b, self.logits)
        # The sampler reads the first 179 columns of each logits row.
        dec = self.decision.index_select(0, order)
        seed = self._seed_value
        sa, sb = self.sample
        act = ext.sample_actions(self.logits, legal_s, order, dec, seed_base=seed, greedy=not sa)[0]
        if sa != sb:
            other = ext.sample_actions(self.logits, legal_s, order, dec, seed_base=seed,
                                       greedy=not sb)[0]
            a_rows = torch.arange(g, device=self.device) < n_a
            act = torch.where(a_rows, act, other)
        actions = torch.empty_like(act)
        actions.index_copy_(0, order, act)
        actions = torch.where(run, actions, -1)
        reward0, new_done, nagari, sstatus = ext.step_indexed(self.states, self.ids, actions)[:4]
        step_ok = sstatus == int(ext.STATUS_OK)
        self.bad[2] += (run & ~step_ok).sum()
        just = run & step_ok & new_done
        self.final_reward0.copy_(torch.where(just, reward0, self.final_reward0))
        self.final_nagari |= just & nagari
        self.steps += run.any().to(torch.int64)
        self.decision += run.to(torch.int32)
        self.running.copy_(run & step_ok & ~new_done)

    def _capture(self) -> None:
        if self._graph is not None and self._graph_sample == self.sample:
            return
        self._graph = None
        # Warm up on a side stream with the state saved and restored around it.
        saved = [t.clone() for t in self._mutable()]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self._step()
        torch.cuda.current_stream().wait_stream(side)
        for t, s in zip(self._mutable(), saved):
            t.copy_(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._step()
        for t, s in zip(self._mutable(), saved):
            t.copy_(s)
        self._graph, self._graph_sample = graph, self.sample

    def _mutable(self) -> list[torch.Tensor]:
        return [self.states, self.running, self.final_reward0, self.final_nagari, self.decision,
                self.bad, self.steps]

    # -- one evaluation --------------------------------------------------------
    def run(self, seed_offset: int, max_steps: int, sample_a: bool = False,
            sample_b: bool = False) -> EvalSummary:
        if max_steps <= 0:
            raise ValueError("max_steps must be positive")
        ext, p, dev = self.ext, self.pairs, self.device
        self.sample = (sample_a, sample_b)
        self._seed_value = seed_offset
        base_seeds, base_first = make_seeds(p, seed_offset, dev)
        self.states.copy_(ext.create(torch.cat((base_seeds, base_seeds)),
                                     torch.cat((base_first, base_first))))
        self.final_reward0.zero_()
        self.final_nagari.zero_()
        self.decision.zero_()
        self.bad.zero_()
        self.steps.zero_()
        # A sampling graph holds the seed it was captured with: recapture on a change.
        if self.graphs and (sample_a or sample_b) and self._graph_seed != seed_offset:
            self._graph = None
        self._graph_seed = seed_offset
        if self.graphs:
            self._capture()
        torch.cuda.synchronize()
        start = time.perf_counter()
        # First observation (python/cugo_eval50.py:193-214): games finished at the
        # deal are excluded; rows that fail to observe are counted and dropped.
        _, legal, _, done, status = ext.observe_indexed_bf16(self.states, self.ids)
        ok = status == int(ext.STATUS_OK)
        has_legal = legal.any(1)
        self.predecision_done.copy_(done)
        self.bad[0] += (~done & ~ok).sum()
        self.bad[1] += (~done & ok & ~has_legal).sum()
        self.running.copy_(~done & ok & has_legal)
        completed = False
        for k in range(max_steps):
            if self.graphs:
                self._graph.replay()
            else:
                self._step()
            if (k + 1) % CHECK_EVERY == 0 or k + 1 == max_steps:
                if not bool(self.running.any()):
                    completed = True
                    break
        torch.cuda.synchronize()
        seconds = time.perf_counter() - start
        observe_bad, legal_bad, step_bad = (int(x) for x in self.bad.tolist())
        if observe_bad:
            raise RuntimeError(f"observe failed on {observe_bad} active visits")
        if legal_bad:
            raise RuntimeError(f"active state had invalid/no legal actions on {legal_bad} visits")
        if step_bad:
            raise RuntimeError(f"step failed on {step_bad} active visits")
        if not completed:
            raise RuntimeError(f"not all games finished within {max_steps} decision steps")
        return summarize(self.final_reward0, self.final_nagari, self.predecision_done,
                         self.a_seat, p, int(self.steps), seconds)

    def release(self) -> None:
        self._graph = None


def summarize(final_reward0: torch.Tensor, final_nagari: torch.Tensor,
              predecision_done: torch.Tensor, a_seat: torch.Tensor, pairs: int,
              decision_steps: int, seconds: float) -> EvalSummary:
    """The statistics of python/cugo_eval50.py:281-361."""
    games = 2 * pairs
    score_a = torch.where(a_seat == 0, final_reward0, -final_reward0)
    p0_score, p1_score = score_a[:pairs], score_a[pairs:]
    pair_score = (p0_score + p1_score) * 0.5

    def wdl(x: torch.Tensor) -> tuple[int, int, int]:
        return int((x > 0).sum().item()), int((x < 0).sum().item()), int((x == 0).sum().item())

    p0_valid = ~predecision_done[:pairs]
    p1_valid = ~predecision_done[pairs:]
    pair_valid = p0_valid & p1_valid
    valid_score = score_a[~predecision_done]
    valid_p0, valid_p1 = p0_score[p0_valid], p1_score[p1_valid]
    valid_pair = pair_score[pair_valid]
    a_wins, b_wins, draws = wdl(valid_score)
    a_p0 = wdl(valid_p0)
    a_p1 = wdl(valid_p1)
    pw = wdl(valid_pair)
    evaluated_pairs = int(pair_valid.sum().item())
    evaluated_games = int((~predecision_done).sum().item())
    mean_pair = float(valid_pair.mean().item()) if evaluated_pairs else 0.0
    if evaluated_pairs > 1:
        pair_std = float(valid_pair.std(unbiased=True).item())
        pair_se = pair_std / math.sqrt(float(evaluated_pairs))
    else:
        pair_std = pair_se = 0.0
    ci_half = 1.959963984540054 * pair_se
    return EvalSummary(
        pairs=pairs, games=games, evaluated_pairs=evaluated_pairs,
        evaluated_games=evaluated_games,
        predecision_excluded=int(predecision_done.sum().item()),
        a_wins=a_wins, b_wins=b_wins, draws=draws,
        a_p0_wins=a_p0[0], a_p0_losses=a_p0[1], a_p0_draws=a_p0[2],
        a_p1_wins=a_p1[0], a_p1_losses=a_p1[1], a_p1_draws=a_p1[2],
        pair_wins=pw[0], pair_losses=pw[1], pair_draws=pw[2],
        mean_score_a=float(valid_score.mean().item()) if evaluated_games else 0.0,
        mean_score_a_p0=float(valid_p0.mean().item()) if valid_p0.numel() else 0.0,
        mean_score_a_p1=float(valid_p1.mean().item()) if valid_p1.numel() else 0.0,
        mean_pair_score_a=mean_pair, pair_score_std=pair_std, pair_score_se=pair_se,
        pair_score_ci95_low=mean_pair - ci_half, pair_score_ci95_high=mean_pair + ci_half,
        terminal=int((~final_nagari).sum().item()), nagari=int(final_nagari.sum().item()),
        decision_steps=decision_steps, seconds=seconds)


def evaluate_paired(ext: Any, model_a: Any, model_b: Any, pairs: int, seed_offset: int,
                    max_steps: int, use_amp: bool = True, sample_a: bool = False,
                    sample_b: bool = False, graphs: bool = True) -> EvalSummary:
    """python/cugo_eval50.py:137-361 (use_amp is accepted for the signature: the
    policies always run in bf16 on the tensor cores)."""
    if pairs <= 0:
        raise ValueError("pairs must be positive")
    if max_steps <= 0:
        raise ValueError("max_steps must be positive")
    ext = ext or load_extension()
    for m in (model_a, model_b):
        if getattr(m, "uses_history", False):
            raise NotImplementedError("sequence policies are not supported by the fused evaluator")
    ev = PairedEvaluator(ext, model_a, model_b, pairs, graphs=graphs)
    try:
        return ev.run(seed_offset, max_steps, sample_a, sample_b)
    finally:
        ev.release()


def match(ext: Any, a: Any, b: Any, pairs: int, chunk: int, seed_offset: int, sample: bool) -> dict:
    """Pooled paired match in chunks (python/league50.py:31-50)."""
    if chunk % 2:
        raise ValueError("chunk must be even so every chunk starts with the same seat order")
    n = total = sq = wins = games = 0
    for start in range(0, pairs, chunk):
        size = min(chunk, pairs - start)
        s = evaluate_paired(ext, a, b, size, chunk_offset(seed_offset, start), max_steps=128,
                            use_amp=True, sample_a=sample, sample_b=sample)
        k = s.evaluated_pairs
        n += k
        total += s.mean_pair_score_a * k
        sq += (s.pair_score_std ** 2) * (k - 1) + k * s.mean_pair_score_a ** 2
        wins += s.a_wins
        games += s.evaluated_games
    mean = total / n
    var = (sq - n * mean ** 2) / (n - 1)
    se = math.sqrt(var / n)
    return {"score": mean, "lo": mean - 1.96 * se, "hi": mean + 1.96 * se,
            "win": 100.0 * wins / games, "pairs": n, "games": games}
