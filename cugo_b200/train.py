"""One PPO iteration of train_ppo50.py on the native kernels: self-play collection
into a device-resident transition store, then the update.  The entry points keep
the reference's names and arguments (python/cugo_ppo50.py: RolloutStorage :273,
collect :321, gae_advantages :484, the update of PpoUpdater :514-745 for the plain
policy target), so train_ppo50.py's loop can call them.

Collection.  The games of an iteration stay in one fixed batch of rows; the running
ones are a device-resident list (rounds.RunningSet) that the step kernel rewrites
every round.  A decision round is:
  observe        bf16 features and legal bit words of the running games
  act            the learner's sampled actions (masked Gumbel-max; one fused
                 kernel for a hidden-512 actor), and in pool games the frozen
                 opponent's actions where it is to move
  record         one kernel appends the round to the store at its device-resident
                 size: features, legal mask, action, log p, the opponent's hand and
                 the next stock draws read from the game row, game and seat, and
                 whether the learner moved
  step           the step kernel with the round's bookkeeping (decision counters,
                 final rewards, the next running list)
With a fused actor nothing in a round waits for the host; the host polls copies of
the running count and of the store size every 4 rounds, and grows the store when a
copy shows it could fill before the next poll.  Opponent rows are dropped from the
store once, after the last round.  Sampling noise is Philox Gumbel noise addressed
by (deal seed, the game's decision count) instead of torch.multinomial: the same
distribution, reproducible.

GAE runs over a dense [sequences, longest] matrix of TD residuals (rows grouped
by (game, seat)), the backward recursion taking one column of every sequence at
a time.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from .evaluate import make_seeds
from .ext import load_extension
from .ppo import GraphedPpoStep, Minibatch, critic_input, make_ppo_step
from .rounds import DONE_BYTE, RunningSet, choose_actions, fused_sampler_params

CHECK_EVERY = 4


@dataclass
class Rollout:
    """python/cugo_ppo50.py:52-66, with the rows' games and seats."""
    features: torch.Tensor  # bf16 [N, 720]
    legal: torch.Tensor     # bool [N, 179]
    actions: torch.Tensor   # int64 [N]
    logp: torch.Tensor      # fp32 [N], behaviour log-prob
    opp_hand: torch.Tensor  # int64 [N]
    stock: torch.Tensor     # int64 [N], the next 8 stock draws (stock_indexed's packing)
    env_ids: torch.Tensor   # int64 [N], the row's game
    seat: torch.Tensor      # int64 [N]
    returns: torch.Tensor   # fp32 [N], scaled final score for the acting player
    games: int
    terminal: int
    nagari: int
    decision_steps: int
    mean_abs_reward0: float
    learner_score: float = float("nan")  # mean scaled score of learner seats in pool games


class RolloutStorage:
    """Device-resident transition store (the reference's RolloutStorage name and
    constructor).  Its size lives in device memory, written by the record kernel
    round by round; `size` is the host copy after a collection.  capacity grows by
    a quarter (at least the needed rows) when a collection would outgrow it."""

    COLUMNS = (("features", torch.bfloat16, 720), ("legal", torch.bool, 179),
               ("actions", torch.int64, 0), ("logp", torch.float32, 0),
               ("opp_hand", torch.int64, 0), ("stock", torch.int64, 0),
               ("env_ids", torch.int64, 0), ("seat", torch.int64, 0),
               ("learner", torch.bool, 0))

    def __init__(self, capacity: int, device: torch.device, all_actions: bool = False) -> None:
        if all_actions:
            raise ValueError("all-action Q targets are not part of this collection")
        self.device = torch.device(device)
        self.all_actions = False
        self.capacity, self.size = 0, 0
        self.sizes = torch.zeros(2, dtype=torch.int64, device=self.device)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.parity = 0
        self.columns: dict[str, torch.Tensor] = {}
        self.reserve(capacity)

    def reserve(self, capacity: int, keep: int = 0) -> None:
        """Reallocates every column with `capacity` rows, keeping the first `keep`."""
        old = self.columns
        self.columns = {}
        for name, dtype, width in self.COLUMNS:
            shape = (capacity, width) if width else (capacity,)
            col = torch.empty(shape, dtype=dtype, device=self.device)
            if keep:
                col[:keep].copy_(old[name][:keep])
            self.columns[name] = col
        self.capacity = capacity

    def clear(self) -> None:
        self.sizes.zero_()
        self.overflow.zero_()
        self.parity, self.size = 0, 0

    def device_size(self) -> torch.Tensor:
        """The size after the last recorded round, int64 [1] in device memory."""
        return self.sizes[self.parity:self.parity + 1]

    def views(self) -> tuple[torch.Tensor, ...]:
        c = self.columns
        return tuple(c[k][:self.size] for k in ("features", "legal", "actions", "logp",
                                                 "opp_hand", "stock", "env_ids", "seat"))


@torch.no_grad()
def collect(ext: Any, actor: nn.Module, pool: list[nn.Module], games: int, seed_offset: int,
            pool_fraction: float, pool_greedy: bool, reward_scale: float,
            storage: RolloutStorage, max_steps: int = 128, critic: nn.Module | None = None,
            **q_options: Any) -> Rollout:
    """Self-play games (seeds make_seeds(games, seed_offset)) recorded into `storage`.

    pool / pool_fraction / pool_greedy: one pool member, drawn for the iteration,
    plays a random seat against the learner in each game with probability
    pool_fraction (greedily or sampled); only the learner's decisions are kept.
    Games that a deal already finished are left out.  A running game without a
    legal action, or a step with a bad status, raises after the collection.
    critic and the all-action options (q_options) belong to the all-action
    targets, which this store does not hold."""
    ext = ext or load_extension()
    dev = torch.device("cuda")
    seeds, first = make_seeds(games, seed_offset, dev)
    states = ext.create(seeds, first)
    opponent = pool[int(torch.randint(len(pool), ()))] if pool and pool_fraction > 0.0 else None
    learner_seat = torch.randint(2, (games,), device=dev)
    vs_pool = (torch.rand(games, device=dev) < pool_fraction) if opponent is not None else None
    started = states[:, DONE_BYTE] == 0
    run = RunningSet(ext, states, started, CHECK_EVERY)
    storage.clear()
    f_actor = fused_sampler_params(actor, 720)
    f_opp = fused_sampler_params(opponent, 720) if opponent is not None else None
    device_count = f_actor is not None and (opponent is None or f_opp is not None)
    actor.eval()
    if opponent is not None:
        opponent.eval()
    while not run.done and run.rounds < max_steps:
        if not device_count and run.read_count() == 0:
            break
        # The store must hold this round's rows: an upper bound of its size is the
        # newest size read back plus a full running set for every round since.
        if device_count:
            size_bound = run.last_seen[1] + (run.rounds - run.last_seen_round) * run.bound
        else:
            size_bound = int(storage.device_size().item())
        if size_bound + run.bound > storage.capacity:
            torch.cuda.synchronize()
            size = int(storage.device_size().item())
            storage.reserve(max(int(storage.capacity * 1.25),
                                size + (CHECK_EVERY * (run.lookahead + 2)) * run.bound), keep=size)
            run.last_seen, run.last_seen_round = (run.last_seen[0], size), run.rounds
        active, count = run.active, run.count
        if not device_count:
            active = active[:run.bound]
        features, bits, players, _, _ = ext.observe_indexed_bf16_bits(
            states, active, m_dev=count if device_count else None)
        actions, logp = choose_actions(ext, actor, f_actor, features, bits, active, seeds,
                                       run.decision, count, False, 0)
        learner = None
        if opponent is not None:
            theirs = choose_actions(ext, opponent, f_opp, features, bits, active, seeds,
                                    run.decision, count, pool_greedy, 1)[0]
            learner = ~vs_pool.index_select(0, active) | (
                players.long() == learner_seat.index_select(0, active))
            actions = torch.where(learner, actions, theirs)
        ext.record_transitions(states, active, count if device_count else None, features, bits,
                               players, actions, logp, learner, storage.sizes, storage.parity,
                               storage.columns, storage.overflow)
        storage.parity ^= 1
        run.step(actions, device_count)
        if device_count and run.poll(storage.device_size()):
            break
    else:
        if not run.done and run.read_count() != 0:
            raise RuntimeError(f"games did not finish within {max_steps} steps")
    storage.size = int(storage.device_size().item())
    if int(storage.overflow.item()):
        raise RuntimeError("transition store overflow")
    if int(run.bad.item()):
        raise RuntimeError("an active game had no legal action, a bad status or a failed step")
    if opponent is not None:  # keep the learner's decisions only, in round order
        keep = torch.nonzero(storage.columns["learner"][:storage.size]).squeeze(1)
        for name, _, _ in RolloutStorage.COLUMNS:
            col = storage.columns[name]
            col[:keep.numel()].copy_(col.index_select(0, keep))
        storage.size = keep.numel()
    features, legal, actions, logp, opp_hand, stock, env_ids, seat = storage.views()
    reward0 = run.reward0
    mine = torch.where(seat == 0, 1.0, -1.0)
    returns = mine * reward0.index_select(0, env_ids) / reward_scale
    n_started = int(started.sum())
    learner_score = float("nan")
    if opponent is not None:
        pool_games = started & vs_pool
        if bool(pool_games.any()):
            own = torch.where(learner_seat == 0, reward0, -reward0)
            learner_score = float(own[pool_games].mean())
    return Rollout(features, legal, actions, logp, opp_hand, stock, env_ids, seat, returns, games,
                   terminal=int((started & ~run.nagari).sum()),
                   nagari=int((started & run.nagari).sum()),
                   decision_steps=int(run.decision.max()) if games else 0,
                   mean_abs_reward0=float(reward0[started].abs().mean()) if n_started else 0.0,
                   learner_score=learner_score)


def gae_advantages(values: torch.Tensor, returns: torch.Tensor, env_ids: torch.Tensor,
                   seat: torch.Tensor, lam: float) -> torch.Tensor:
    """GAE(lambda), gamma 1, over each (game, seat) sequence of own decisions (the
    reference's definition, python/cugo_ppo50.py:484-509): residual_t = V(the seat's
    next decision) - V(t), or return - V(t) at the seat's last decision;
    A_t = residual_t + lam * A_(t+1) within the sequence; lam >= 1 gives return - V.
    Rows must be in decision order within each sequence (as collect stores them).

    The sequences are laid out as the rows of a dense [sequences, longest] matrix
    of residuals (a stable sort groups each sequence's rows in order; a row's column
    is its index in the sequence, padding is zero), the recursion runs backwards
    over the columns on all sequences at once, and each row reads its entry back."""
    if lam >= 1.0:
        return returns - values
    n = values.numel()
    if n == 0:
        return values.clone()
    dev = values.device
    key = env_ids * 2 + seat
    order = torch.sort(key, stable=True).indices
    k = key.index_select(0, order)
    v = values.index_select(0, order).float()
    last = torch.ones(n, dtype=torch.bool, device=dev)
    last[:-1] = k[1:] != k[:-1]
    nxt = torch.cat((v[1:], v[:1]))
    resid = torch.where(last, returns.index_select(0, order).float(), nxt) - v
    head = torch.ones(n, dtype=torch.bool, device=dev)
    head[1:] = last[:-1]
    idx = torch.arange(n, device=dev)
    col = idx - torch.where(head, idx, 0).cummax(0).values
    seq = torch.cumsum(head.long(), 0) - 1
    width = int(col.max()) + 1
    dense = torch.zeros((int(seq[-1]) + 1, width + 1), dtype=torch.float32, device=dev)
    dense[seq, col] = resid
    for c in range(width - 1, -1, -1):
        dense[:, c].add_(dense[:, c + 1], alpha=lam)
    out = torch.empty_like(values)
    out[order] = dense[seq, col].to(values.dtype)
    return out


@dataclass
class TrainStats:
    """python/cugo_ppo50.py:460-476 (the plain-target fields).  With several ranks
    the statistics cover every rank's rows (sums all-reduced)."""
    policy_loss: float
    value_loss: float
    entropy: float
    kl: float
    clipfrac: float
    explained_var: float
    updates: int
    epochs: float
    belief_loss: float = float("nan")


class PpoTrainer:
    """The update of one iteration (python/cugo_ppo50.py:514-745, PpoUpdater.update with
    the plain policy target) over the fused networks.

    Data parallel (world > 1, one process per GPU, process group initialised): each
    rank updates on its own rollout and PpoStep averages the gradients.  The ranks
    must take the same collective steps, so every epoch runs the smallest number of
    whole minibatches any rank has, and the early stop compares the KL averaged over
    the ranks."""

    def __init__(self, actor: nn.Module, critic: nn.Module, lr: float = 3e-4,
                 minibatch: int = 32768, clip: float = 0.2, value_coef: float = 0.5,
                 grad_clip: float = 1.0, use_graph: bool = True, world: int = 1,
                 belief: nn.Module | None = None, belief_coef: float = 0.0) -> None:
        self.actor, self.critic, self.minibatch = actor, critic, minibatch
        self.belief = belief
        params = list(actor.parameters()) + list(critic.parameters())
        params += list(belief.parameters()) if belief is not None else []
        # The reference trainer's optimizer (python/train_ppo50.py:153-156).
        self.optimizer = torch.optim.Adam(params, lr=lr, eps=1e-5, fused=True, capturable=use_graph)
        self.step = make_ppo_step(actor, critic, self.optimizer, clip, value_coef, grad_clip, world,
                                  belief, belief_coef)
        self.use_graph = use_graph
        self.world = world
        self.graphed: GraphedPpoStep | None = None

    def _reduce(self, t: torch.Tensor, op=None) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, op=op or dist.ReduceOp.SUM)
        return t

    def _steps_per_epoch(self, n: int, device: torch.device) -> int:
        t = torch.tensor([n // self.minibatch], dtype=torch.int64, device=device)
        return int(self._reduce(t, dist.ReduceOp.MIN if self.world > 1 else None))

    def _kl(self) -> float:
        kl = self._reduce(self.step.last_kl.detach().reshape(1).clone())
        return float(kl) / self.world

    @torch.no_grad()
    def values(self, data: Rollout, chunk: int = 65536) -> torch.Tensor:
        self.critic.eval()
        n = data.actions.numel()
        if n == 0:
            return torch.zeros(0, device=data.returns.device)
        stock = data.stock if getattr(self.critic, "stock", False) else None
        parts = [self.critic(critic_input(data.features[i:i + chunk], data.opp_hand[i:i + chunk],
                                          None if stock is None else stock[i:i + chunk]))
                 for i in range(0, n, chunk)]
        if getattr(self.critic, "value_bins", 0):  # the mean of the return distribution
            return torch.cat([self.critic.value(p) for p in parts])
        return torch.cat([p.float().reshape(-1) for p in parts])

    def _explained_variance(self, returns: torch.Tensor, values: torch.Tensor) -> float:
        """1 - Var(return - V) / Var(return), over every rank's rows."""
        r, e = returns.double(), (returns - values).double()
        m = torch.stack((torch.tensor(float(r.numel()), dtype=torch.float64, device=r.device),
                         r.sum(), (r * r).sum(), e.sum(), (e * e).sum()))
        n, rs, rq, es, eq = self._reduce(m).tolist()
        if n < 2:
            return float("nan")
        var_r = (rq - rs * rs / n) / (n - 1)
        var_e = (eq - es * es / n) / (n - 1)
        return 1.0 - var_e / max(var_r, 1e-8)

    def update(self, data: Rollout, epochs: int, entropy_coef: float, target_kl: float,
               gae_lambda: float = 1.0) -> TrainStats:
        n = data.actions.numel()
        values = self.values(data)
        adv = gae_advantages(values, data.returns, data.env_ids, data.seat, gae_lambda)
        ret = adv + values
        explained_var = self._explained_variance(data.returns, values)
        self.actor.train()
        self.critic.train()
        st = self.step
        st.entropy_coef.fill_(entropy_coef)
        st.sums.zero_()
        updates, stop = 0, False
        steps = self._steps_per_epoch(n, data.actions.device)
        with_stock = bool(getattr(self.critic, "stock", False))
        for _ in range(epochs):
            perm = torch.randperm(n, device=data.actions.device)
            for j in range(steps):
                idx = perm[j * self.minibatch:(j + 1) * self.minibatch]
                mb = Minibatch(data.features.index_select(0, idx), data.legal.index_select(0, idx),
                               data.actions.index_select(0, idx), data.logp.index_select(0, idx),
                               data.opp_hand.index_select(0, idx), adv.index_select(0, idx),
                               ret.index_select(0, idx),
                               data.stock.index_select(0, idx) if with_stock else None)
                if self.use_graph:
                    if self.graphed is None:
                        self.graphed = GraphedPpoStep(st, mb)
                    self.graphed(mb)
                else:
                    st.step(mb)
                updates += 1
                if target_kl > 0 and updates % 8 == 0 and self._kl() > 1.5 * target_kl:
                    stop = True
                    break
            if stop:
                break
        s = self._reduce(st.sums.detach().double().clone()).tolist()
        count = max(1.0, s[5])
        return TrainStats(policy_loss=s[0] / count, value_loss=s[1] / count, entropy=s[2] / count,
                          kl=s[3] / count, clipfrac=s[4] / count, explained_var=explained_var,
                          updates=updates, epochs=updates / max(1, steps),
                          belief_loss=s[6] / count if self.belief is not None else float("nan"))


def iteration(ext: Any, trainer: PpoTrainer, storage: RolloutStorage, games: int,
              seed_offset: int, reward_scale: float = 32.0, epochs: int = 2,
              entropy_coef: float = 0.05, target_kl: float = 0.03,
              gae_lambda: float = 0.95, pool: list[nn.Module] | None = None,
              pool_fraction: float = 0.0, pool_greedy: bool = False) -> dict:
    """One train_ppo50.py iteration (its defaults: 65,536 games, 2 epochs, minibatch
    32,768, GAE 0.95, reward scale 32): collection and update, timed on the host
    around device synchronisations.  Data parallel: each rank passes its own
    seed_offset (disjoint games) and a trainer built with world = the number of ranks."""
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    data = collect(ext, trainer.actor, pool or [], games, seed_offset, pool_fraction, pool_greedy,
                   reward_scale, storage)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    stats = trainer.update(data, epochs, entropy_coef, target_kl, gae_lambda)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    return dict(collect_seconds=t1 - t0, update_seconds=t2 - t1, seconds=t2 - t0,
                rows=int(data.actions.numel()), games=games, decision_steps=data.decision_steps,
                stats=stats)
