"""All-action and redealt-world branching on the native kernels: the value estimates
of the reference's all-action PPO mode (python/cugo_ppo50.py:84-270), same names,
arguments and results.

  action_values   Q of every marked action: branch the row with the action
                  (branch_indexed), observe the child with the critic's input
                  written in the same pass (observe_critic_bf16: features and the
                  hand plane of the mover's opponent), score it with the critic on
                  the fused GEMM; a finished child scores its final reward.
  redeal_worlds   copies of rows in which the observer's opponent holds another
                  hand consistent with everything the observer saw, kept when the
                  observer's features and legal actions are unchanged: redeal,
                  observe and compare run on the device in one launch
                  (cugo_b200_redeal_worlds).
  world_values    Q averaged over redealt worlds, each child scored by the critic
                  (depth 1) or by greedy play to the end (depth 0).

The random source of the redeal is Philox (seed, attempt) instead of torch's
generator, so the worlds are reproducible; the critic takes the features and the
opponent's hand (the stock planes of OracleCritic(stock=True) are not written by
the fused observe and are refused).
"""
from __future__ import annotations

from typing import Any

import torch
from torch import nn

from .ext import load_extension

Q_CHUNK = 65536      # children per critic pass (python/cugo_ppo50.py:84)
ROLLOUT_STEPS = 96   # python/cugo_ppo50.py:114
ROLLOUT_CHECK = 4    # python/cugo_ppo50.py:180
CRITIC_LD = 776      # 720 features + 50 hand bits, rows padded to 16 bytes


def _chunk(net: nn.Module | None) -> int:
    """Children per critic pass: Q_CHUNK at the reference's 2,048-wide hidden layer,
    proportionally more for narrower networks (the same activation memory, fewer
    host round trips)."""
    inp = getattr(net, "inp", None)
    hidden = getattr(inp, "out_features", 2048) if inp is not None else 2048
    return Q_CHUNK * max(1, 2048 // max(1, hidden))


def _critic_rows(ext: Any, critic: nn.Module, child: torch.Tensor):
    """Critic values of the children and the mover of each (python/cugo_ppo50.py:97-101)."""
    if getattr(critic, "stock", False):
        raise RuntimeError("the fused critic input carries no stock planes (critic.stock must be False)")
    ids = torch.arange(child.shape[0], device=child.device)
    crit_in, players, _, _ = ext.observe_critic_bf16(child, ids, width=CRITIC_LD)
    out = critic(crit_in)
    value = getattr(critic, "value", None)
    v = value(out) if callable(value) else out.float().reshape(-1)
    return v, players.to(torch.int64)


@torch.no_grad()
def action_values(ext: Any, critic: nn.Module, states: torch.Tensor, env_rows: torch.Tensor,
                  seat: torch.Tensor, branch: torch.Tensor, reward_scale: float) -> torch.Tensor:
    """[R, 179] fp16 Q for the player to move of each action marked in `branch`
    (NaN elsewhere) -- python/cugo_ppo50.py:87-104."""
    ext = ext or load_extension()
    rows, acts = torch.nonzero(branch, as_tuple=True)
    q = torch.full(branch.shape, float("nan"), dtype=torch.float16, device=branch.device)
    me = seat.index_select(0, rows)
    chunk = _chunk(critic)
    for i in range(0, rows.numel(), chunk):
        r, a, m = rows[i:i + chunk], acts[i:i + chunk], me[i:i + chunk]
        child, reward0, done = ext.branch_indexed(states, env_rows.index_select(0, r), a)[:3]
        v, mover = _critic_rows(ext, critic, child)
        v = torch.where(mover == m, v, -v)  # zero-sum: the opponent's value is ours negated
        final = torch.where(m == 0, reward0, -reward0) / reward_scale
        q[r, a] = torch.where(done, final, v).to(torch.float16)
    return q


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


def _greedy(ext: Any, model: nn.Module, features: torch.Tensor, legal: torch.Tensor,
            ids: torch.Tensor, zeros: torch.Tensor) -> torch.Tensor:
    """Masked argmax of the model's logits, lowest action on ties (the reference's
    _act(..., greedy=True), python/cugo_ppo50.py:73-82), in the sampler kernel."""
    out = model(features)
    logits = (out[0] if isinstance(out, tuple) else out).float()
    return ext.sample_actions(logits, legal, ids, zeros[:ids.numel()], greedy=True)[0]


@torch.no_grad()
def greedy_to_end(ext: Any, actor: nn.Module, opponent: nn.Module | None, child: torch.Tensor,
                  reward0: torch.Tensor, done: torch.Tensor, me: torch.Tensor,
                  pool: torch.Tensor) -> torch.Tensor:
    """Final score (seat 0) of each child after greedy play to the end; in pool games
    the opponent network plays the seat that is not `me`
    (python/cugo_ppo50.py:183-211).  Finished games keep reporting their final
    score, so the batch keeps its shape for ROLLOUT_CHECK steps between host reads
    and is compacted only when under 60% of it is still running."""
    ext = ext or load_extension()
    final = torch.where(done, reward0, 0.0)
    ids = torch.nonzero(~done).squeeze(1)
    zeros = torch.zeros(child.shape[0], dtype=torch.int32, device=child.device)
    steps = 0
    while ids.numel():
        pool_rows = torch.nonzero(pool.index_select(0, ids)).squeeze(1) if opponent is not None else None
        pool_me = me.index_select(0, ids).index_select(0, pool_rows) if pool_rows is not None else None
        for _ in range(ROLLOUT_CHECK):
            features, legal, players = ext.observe_indexed_bf16(child, ids)[:3]
            step = _greedy(ext, actor, features, legal, ids, zeros)
            if pool_rows is not None and pool_rows.numel():
                f, l = features.index_select(0, pool_rows), legal.index_select(0, pool_rows)
                theirs = players.index_select(0, pool_rows).to(torch.int64) != pool_me
                mine = step.index_select(0, pool_rows)
                step.index_copy_(0, pool_rows, torch.where(
                    theirs, _greedy(ext, opponent, f, l, ids.index_select(0, pool_rows), zeros), mine))
            reward, new_done = ext.step_indexed(child, ids, step)[:2]
            final.index_copy_(0, ids, reward)
        steps += ROLLOUT_CHECK
        running = int((~new_done).sum())
        if running == 0:
            break
        if steps >= ROLLOUT_STEPS:
            raise RuntimeError(f"rollout did not finish within {ROLLOUT_STEPS} steps")
        if running < 0.6 * ids.numel():
            ids = ids.index_select(0, torch.nonzero(~new_done).squeeze(1))
    return final


@torch.no_grad()
def child_values(ext: Any, critic: nn.Module, child: torch.Tensor, reward0: torch.Tensor,
                 done: torch.Tensor, me: torch.Tensor, reward_scale: float) -> torch.Tensor:
    """Scaled value for `me` of each child one step in: its final score, else the
    critic (python/cugo_ppo50.py:214-225)."""
    ext = ext or load_extension()
    v, mover = _critic_rows(ext, critic, child)
    v = torch.where(mover == me, v, -v)
    return torch.where(done, torch.where(me == 0, reward0, -reward0) / reward_scale, v)


def _world_q(ext: Any, actor: nn.Module, opponent: nn.Module | None, critic: nn.Module | None,
             states: torch.Tensor, env_rows: torch.Tensor, seat: torch.Tensor, vs_pool: torch.Tensor,
             branch: torch.Tensor, reward_scale: float, worlds: int, depth: int,
             seed: int) -> torch.Tensor:
    """[worlds, R, 179] fp32 Q per redealt world, 0 where not branched
    (python/cugo_ppo50.py:228-243)."""
    w = redeal_worlds(ext, states, env_rows, seat, worlds, seed=seed)
    seat_k, pool_k, branch_k = seat.repeat(worlds), vs_pool.repeat(worlds), branch.repeat(worlds, 1)
    rows, acts = torch.nonzero(branch_k, as_tuple=True)
    q = torch.zeros(branch_k.shape, device=branch.device)
    chunk = _chunk(critic if depth == 1 else actor)
    for i in range(0, rows.numel(), chunk):
        r, a = rows[i:i + chunk], acts[i:i + chunk]
        me, pool = seat_k.index_select(0, r), pool_k.index_select(0, r)
        child, reward0, done = ext.branch_indexed(w, r, a)[:3]
        if depth == 1:
            q[r, a] = child_values(ext, critic, child, reward0, done, me, reward_scale)
        else:
            final = greedy_to_end(ext, actor, opponent, child, reward0, done, me, pool)
            q[r, a] = torch.where(me == 0, final, -final) / reward_scale
    return q.view(worlds, *branch.shape)


@torch.no_grad()
def world_values(ext: Any, actor: nn.Module, opponent: nn.Module | None, states: torch.Tensor,
                 env_rows: torch.Tensor, seat: torch.Tensor, vs_pool: torch.Tensor,
                 branch: torch.Tensor, reward_scale: float, worlds: int,
                 critic: nn.Module | None = None, depth: int = 0, first: int = 0,
                 seed: int = 0) -> torch.Tensor:
    """[R, 179] fp16 Q of each branched action averaged over redealt worlds (NaN
    elsewhere) -- python/cugo_ppo50.py:246-270.  depth 0 plays each branch to the
    end, depth 1 scores the child with the critic in that world; first > 0 deals
    that many worlds and the rest only to decisions whose best action differs
    between them."""
    ext = ext or load_extension()
    args = (ext, actor, opponent, critic)
    if 0 < first < worlds:
        q = _world_q(*args, states, env_rows, seat, vs_pool, branch, reward_scale, first, depth, seed)
        best = q.masked_fill(~branch, float("-inf")).argmax(-1)
        total = q.sum(0)
        count = torch.full((branch.shape[0], 1), float(first), device=branch.device)
        rows = torch.nonzero((best != best[:1]).any(0)).squeeze(1)
        if rows.numel():
            more = _world_q(*args, states, env_rows.index_select(0, rows), seat.index_select(0, rows),
                            vs_pool.index_select(0, rows), branch.index_select(0, rows),
                            reward_scale, worlds - first, depth, seed + 1)
            total.index_add_(0, rows, more.sum(0))
            count.index_fill_(0, rows, float(worlds))
        q = total / count
    else:
        q = _world_q(*args, states, env_rows, seat, vs_pool, branch, reward_scale, worlds, depth,
                     seed).mean(0)
    return torch.where(branch, q, float("nan")).to(torch.float16)
