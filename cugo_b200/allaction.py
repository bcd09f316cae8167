"""All-action and redealt-world value estimates on the native kernels: the values the
reference's all-action PPO mode trains against (python/cugo_ppo50.py:84-270), with
its entry points' names, arguments and results (action_values, redeal_worlds,
world_values; greedy_to_end and child_values for its _greedy_to_end and
_child_values).

How the work is laid out here:

  branch pairs   every marked (decision row, action) pair, row-major, is one child;
                 children are made (branch_indexed) and valued in fixed-size chunks,
                 and a chunk's values land in the flat [rows x 179] result at
                 row * 179 + action
  critic input   observe_critic_bf16 writes the critic's whole input row in the
                 observe pass (the mover's features and the hand plane of the mover's
                 opponent; with a stock critic, stock_planes_bf16 then sets the
                 one-hot planes of the next 8 stock draws in the same rows)
  values         a child that ended the game is worth its final score for the
                 decision's player; otherwise the critic's value, negated when the
                 opponent moves next (zero sum)
  greedy play    children play to the end in a device-resident running set
                 (rounds.RunningSet): per round observe, the actor's greedy action
                 (the fused policy kernel in greedy mode where it runs the actor),
                 the pool opponent's where it is to move, and the step with the
                 round's bookkeeping; finished children keep their final reward and
                 nothing is compacted on the host
  worlds         redeal_worlds deals, observes and accepts every world row in one
                 launch (cugo_b200_redeal_worlds); world k is valued like the real
                 deal and the values are averaged

The redeal draws from Philox (seed, attempt, world row) instead of torch's
generator, so the worlds are reproducible.
"""
from __future__ import annotations

from typing import Any

import torch
from torch import nn

from .ext import load_extension
from .rounds import RunningSet, choose_actions, fused_sampler_params

Q_CHUNK = 65536      # children per pass at a 2,048-wide critic (python/cugo_ppo50.py:84)
ROLLOUT_STEPS = 96   # decisions a greedy rollout may take (python/cugo_ppo50.py:114)
ACTIONS = 179
CRITIC_WIDTH = 776   # 720 features + 50 hand bits, rows padded to 16 bytes
STOCK_WIDTH = 1176   # ... + 400 stock planes (8 draws x 50 cards)


def _children_per_pass(net: nn.Module | None) -> int:
    """Q_CHUNK scaled up for narrower networks (the same activation memory per pass)."""
    hidden = 2048
    inp = getattr(net, "inp", None)
    if inp is not None:
        hidden = max(1, getattr(inp, "out_features", 2048))
    return Q_CHUNK * max(1, 2048 // hidden)


def _pairs(branch: torch.Tensor):
    """Row-major (row, action) pairs of the marked entries of a [R, 179] mask."""
    flat = torch.nonzero(branch.reshape(-1)).squeeze(1)
    return flat, flat // branch.shape[1], flat % branch.shape[1]


def _critic_values(ext: Any, critic: nn.Module, children: torch.Tensor):
    """(critic value of each child for its mover, the mover)."""
    ids = torch.arange(children.shape[0], device=children.device)
    stock = bool(getattr(critic, "stock", False))
    rows, movers, _, _ = ext.observe_critic_bf16(children, ids,
                                                 width=STOCK_WIDTH if stock else CRITIC_WIDTH)
    if stock:
        ext.stock_planes_bf16(children, ids, rows, first_column=770)
    out = critic(rows)
    head = getattr(critic, "value", None)
    value = head(out) if callable(head) else out.float().reshape(-1)
    return value, movers.long()


def _for_player(value: torch.Tensor, mover: torch.Tensor, player: torch.Tensor) -> torch.Tensor:
    """A mover's value seen by `player` (zero sum)."""
    return torch.where(mover == player, value, -value)


def _final_for(reward0: torch.Tensor, player: torch.Tensor, scale: float) -> torch.Tensor:
    """Player 0's final reward seen by `player`, scaled."""
    return torch.where(player == 0, reward0, -reward0) / scale


@torch.no_grad()
def child_values(ext: Any, critic: nn.Module, child: torch.Tensor, reward0: torch.Tensor,
                 done: torch.Tensor, me: torch.Tensor, reward_scale: float) -> torch.Tensor:
    """Scaled value for `me` of each child one step in: its final score, else the
    critic (python/cugo_ppo50.py:214-225)."""
    ext = ext or load_extension()
    value, mover = _critic_values(ext, critic, child)
    return torch.where(done, _final_for(reward0, me, reward_scale), _for_player(value, mover, me))


@torch.no_grad()
def action_values(ext: Any, critic: nn.Module, states: torch.Tensor, env_rows: torch.Tensor,
                  seat: torch.Tensor, branch: torch.Tensor, reward_scale: float) -> torch.Tensor:
    """[R, 179] fp16 Q, for the player to move, of each action marked in `branch`
    (NaN elsewhere) -- python/cugo_ppo50.py:87-104."""
    ext = ext or load_extension()
    q = torch.full((branch.numel(),), float("nan"), dtype=torch.float16, device=branch.device)
    flat, rows, acts = _pairs(branch)
    per_pass = _children_per_pass(critic)
    for lo in range(0, flat.numel(), per_pass):
        part = slice(lo, lo + per_pass)
        child, reward0, done = ext.branch_indexed(states, env_rows.index_select(0, rows[part]),
                                                  acts[part])[:3]
        who = seat.index_select(0, rows[part])
        q[flat[part]] = child_values(ext, critic, child, reward0, done, who,
                                     reward_scale).to(torch.float16)
    return q.view(branch.shape)


@torch.no_grad()
def redeal_worlds(ext: Any, states: torch.Tensor, env_rows: torch.Tensor, seat: torch.Tensor,
                  worlds: int, tries: int = 8, seed: int = 0) -> torch.Tensor:
    """[worlds * R, 248] copies of the rows, world-major, each redealt so the
    observer's features and legal actions are unchanged; a row that fails `tries`
    times keeps the real deal (python/cugo_ppo50.py:152-177).  One kernel launch
    (cugo_b200_redeal_worlds) runs the attempts of every world row; attempt t of
    world row w draws from Philox (seed, t, w)."""
    ext = ext or load_extension()
    if states.shape[1] != ext.STATE_BYTES:
        raise RuntimeError("state rows must be TorchEnv50 images")
    return ext.redeal_worlds(states, env_rows, seat, worlds, seed=seed, tries=tries)


def _greedy_actions(ext: Any, model: nn.Module, features, bits, rows, count, decision, positions):
    """The model's masked argmax (lowest action on ties, the reference's greedy _act,
    python/cugo_ppo50.py:73-82) for the running rows (positions: the batch's row
    numbers, which stand in for the noise address greedy play does not use)."""
    fused = fused_sampler_params(model, features.shape[1])
    return choose_actions(ext, model, fused, features, bits, rows, positions, decision, count, True,
                          0)[0]


@torch.no_grad()
def greedy_to_end(ext: Any, actor: nn.Module, opponent: nn.Module | None, child: torch.Tensor,
                  reward0: torch.Tensor, done: torch.Tensor, me: torch.Tensor,
                  pool: torch.Tensor) -> torch.Tensor:
    """Player 0's final score of each child after greedy play to the end; in pool
    games (pool[i]) the opponent network plays the seat that is not me[i]
    (python/cugo_ppo50.py:183-211).  Children that already ended keep reward0."""
    ext = ext or load_extension()
    run = RunningSet(ext, child, ~done)
    rivals = opponent is not None and bool(pool.any())
    device_count = fused_sampler_params(actor, 720) is not None and (
        not rivals or fused_sampler_params(opponent, 720) is not None)
    while not run.done and run.rounds < ROLLOUT_STEPS:
        if not device_count and run.read_count() == 0:
            break
        active, count = run.active, run.count
        if not device_count:
            active = active[:run.bound]
        features, bits, players, _, _ = ext.observe_indexed_bf16_bits(
            child, active, m_dev=count if device_count else None)
        actions = _greedy_actions(ext, actor, features, bits, active, count, run.decision,
                                  run.positions)
        if rivals:
            theirs = _greedy_actions(ext, opponent, features, bits, active, count, run.decision,
                                     run.positions)
            rival_moves = pool.index_select(0, active) & (players.long() != me.index_select(0, active))
            actions = torch.where(rival_moves, theirs, actions)
        run.step(actions, device_count)
        if device_count:
            run.poll()
    if not run.done and run.read_count() != 0:
        raise RuntimeError(f"rollout did not finish within {ROLLOUT_STEPS} steps")
    if int(run.bad.item()):
        raise RuntimeError("a greedy rollout met a bad status")
    return torch.where(done, reward0, run.reward0)


def _world_pass(ext: Any, actor, opponent, critic, worlds_rows: torch.Tensor, world_rows: torch.Tensor,
                seat: torch.Tensor, vs_pool: torch.Tensor, branch: torch.Tensor,
                reward_scale: float, depth: int, out: torch.Tensor) -> None:
    """Adds each branched action's value in one set of world rows into out [R, 179]
    (fp32): world_rows[i] is row i's copy in worlds_rows."""
    flat, rows, acts = _pairs(branch)
    per_pass = _children_per_pass(critic if depth == 1 else actor)
    acc = out.view(-1)
    for lo in range(0, flat.numel(), per_pass):
        part = slice(lo, lo + per_pass)
        r = rows[part]
        who = seat.index_select(0, r)
        child, reward0, done = ext.branch_indexed(worlds_rows, world_rows.index_select(0, r),
                                                  acts[part])[:3]
        if depth == 1:
            v = child_values(ext, critic, child, reward0, done, who, reward_scale)
        else:
            final = greedy_to_end(ext, actor, opponent, child, reward0, done, who,
                                  vs_pool.index_select(0, r))
            v = _final_for(final, who, reward_scale)
        acc.index_add_(0, flat[part], v.float())


@torch.no_grad()
def world_values(ext: Any, actor: nn.Module, opponent: nn.Module | None, states: torch.Tensor,
                 env_rows: torch.Tensor, seat: torch.Tensor, vs_pool: torch.Tensor,
                 branch: torch.Tensor, reward_scale: float, worlds: int,
                 critic: nn.Module | None = None, depth: int = 0, first: int = 0,
                 seed: int = 0) -> torch.Tensor:
    """[R, 179] fp16 Q of each branched action averaged over redealt worlds (NaN
    elsewhere) -- python/cugo_ppo50.py:246-270.  depth 0 plays each branch to the
    end, depth 1 scores the child with the critic in that world.  0 < first <
    worlds: `first` worlds (seed) for every decision, the other worlds - first
    (seed + 1) only for decisions whose best action differs between those first."""
    ext = ext or load_extension()
    r = branch.shape[0]
    dev = branch.device
    staged = 0 < first < worlds
    n0 = first if staged else worlds
    total = torch.zeros(branch.shape, device=dev)
    counts = torch.full((r, 1), float(n0), device=dev)
    base = redeal_worlds(ext, states, env_rows, seat, n0, seed=seed)
    best = []
    for k in range(n0):
        q_k = torch.zeros(branch.shape, device=dev)
        _world_pass(ext, actor, opponent, critic, base, torch.arange(r, device=dev) + k * r, seat,
                    vs_pool, branch, reward_scale, depth, q_k)
        total += q_k
        if staged:
            best.append(q_k.masked_fill(~branch, float("-inf")).argmax(1))
    if staged:
        best = torch.stack(best)
        open_rows = torch.nonzero((best != best[:1]).any(0)).squeeze(1)
        if open_rows.numel():
            more = worlds - first
            extra = redeal_worlds(ext, states, env_rows.index_select(0, open_rows),
                                  seat.index_select(0, open_rows), more, seed=seed + 1)
            sub = branch.index_select(0, open_rows)
            n_open = open_rows.numel()
            acc = torch.zeros(sub.shape, device=dev)
            for k in range(more):
                _world_pass(ext, actor, opponent, critic, extra,
                            torch.arange(n_open, device=dev) + k * n_open,
                            seat.index_select(0, open_rows), vs_pool.index_select(0, open_rows),
                            sub, reward_scale, depth, acc)
            total.index_add_(0, open_rows, acc)
            counts.index_fill_(0, open_rows, float(worlds))
    return torch.where(branch, total / counts, float("nan")).to(torch.float16)
