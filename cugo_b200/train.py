"""One PPO iteration of train_ppo50.py on the native kernels: self-play collection with
recorded transitions, then the update (python/cugo_ppo50.py:321-450 collect,
:484-509 gae_advantages, :514-745 PpoUpdater.update), same arguments and results
for the plain policy target.

collect    every decision round observes the running games (bf16 features, bool legal
           masks), runs the actor and samples its action in one fused kernel where the
           actor is a hidden-512 FusedResidualMlp (masked Gumbel-max from Philox
           instead of torch.multinomial over the softmax: the same distribution,
           reproducible), records features, legal mask, action, behaviour log p, the
           opponent's hand, game and seat, and steps the games; the returns are the
           final scores from each row's seat, divided by reward_scale.
update     critic values of every row (the fused inference path), GAE(lambda) along
           each (game, seat) sequence, then `epochs` passes of shuffled minibatches
           through the PPO step captured as a CUDA graph (GraphedPpoStep), stopping
           early when the minibatch KL exceeds 1.5 x target_kl (checked every 8).
The pool opponent, all-action Q targets and belief head of the reference are not
part of this iteration.
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
from .ppo import GraphedPpoStep, Minibatch, PpoStep, critic_input


@dataclass
class Rollout:
    """python/cugo_ppo50.py:52-66 (without the stock planes and pool statistics)."""
    features: torch.Tensor  # bf16 [N, 720]
    legal: torch.Tensor     # bool [N, 179]
    actions: torch.Tensor   # int64 [N]
    logp: torch.Tensor      # fp32 [N], behaviour log-prob
    opp_hand: torch.Tensor  # int64 [N]
    env_ids: torch.Tensor   # int64 [N], the row's game
    seat: torch.Tensor      # int64 [N]
    returns: torch.Tensor   # fp32 [N], scaled final score for the acting player
    games: int
    terminal: int
    nagari: int
    decision_steps: int
    mean_abs_reward0: float


class RolloutStorage:
    """Fixed transition buffers reused every iteration, grown by a quarter when a
    collection outgrows them (python/cugo_ppo50.py:273-318)."""

    def __init__(self, capacity: int, device: torch.device) -> None:
        self.device, self.size, self.capacity = device, 0, 0
        self.tensors: tuple[torch.Tensor, ...] = ()
        self._allocate(capacity)

    def _allocate(self, capacity: int) -> None:
        d, old = self.device, self.tensors
        self.tensors = (
            torch.empty((capacity, 720), dtype=torch.bfloat16, device=d),
            torch.empty((capacity, 179), dtype=torch.bool, device=d),
            torch.empty(capacity, dtype=torch.int64, device=d),
            torch.empty(capacity, dtype=torch.float32, device=d),
            torch.empty(capacity, dtype=torch.int64, device=d),
            torch.empty(capacity, dtype=torch.int64, device=d),
            torch.empty(capacity, dtype=torch.int64, device=d),
        )
        for new_t, old_t in zip(self.tensors, old):
            new_t[:self.size].copy_(old_t[:self.size])
        self.capacity = capacity

    def append(self, *parts: torch.Tensor) -> None:
        n = parts[0].shape[0]
        if self.size + n > self.capacity:
            self._allocate(int((self.size + n) * 1.25))
        for t, part in zip(self.tensors, parts):
            t[self.size:self.size + n].copy_(part)
        self.size += n

    def views(self) -> tuple[torch.Tensor, ...]:
        return tuple(t[:self.size] for t in self.tensors)


def _act_sample(ext: Any, actor: nn.Module, features: torch.Tensor, legal: torch.Tensor,
                game: torch.Tensor, decision: torch.Tensor, seed_base: int):
    """Sampled actions and their log-probabilities under the actor: one fused launch
    for a hidden-512 FusedResidualMlp, else the actor's forward and the sampler."""
    from .policy import fused_mlp_supported
    infer = getattr(actor, "_weights", None)
    if infer is not None:
        params = [t for l in actor.linears() for t in (l.weight, l.bias)]
        ws, bs = actor._weights(params)
        if fused_mlp_supported(ws[0].shape[0], actor.n_blocks, ws[0].shape[1], ws[-1].shape[0]) \
                and ws[-1].shape[0] >= 179 and ws[0].shape[1] == features.shape[1]:
            from .ppo import _ACT
            actions, logp, _ = ext.mlp_fused_sample(features, ws, bs, _ACT[actor.activation],
                                                    ext.pack_legal(legal), game, decision,
                                                    seed_base)
            return actions, logp
    out = actor(features)
    logits = (out[0] if isinstance(out, tuple) else out).float().contiguous()
    return ext.sample_actions(logits, legal, game, decision, seed_base)


@torch.no_grad()
def collect(ext: Any, actor: nn.Module, games: int, seed_offset: int, reward_scale: float,
            storage: RolloutStorage, max_steps: int = 128) -> Rollout:
    """Self-play games with recorded transitions (python/cugo_ppo50.py:321-450,
    without pool opponents): seeds make_seeds(games, seed_offset); games finished
    before any decision are left out; a bad status or a running game without a
    legal action raises."""
    ext = ext or load_extension()
    device = torch.device("cuda")
    seeds, first = make_seeds(games, seed_offset, device)
    states = ext.create(seeds, first)
    final_reward0 = torch.zeros(games, device=device)
    final_nagari = torch.zeros(games, dtype=torch.bool, device=device)
    started = torch.zeros(games, dtype=torch.bool, device=device)
    active = torch.arange(games, device=device)
    storage.size = 0
    steps = 0
    bad = torch.zeros((), dtype=torch.int64, device=device)
    actor.eval()
    for _ in range(max_steps):
        features, legal, players, done, status = ext.observe_indexed_bf16(states, active)
        keep = ~done & (status == int(ext.STATUS_OK)) & legal.any(dim=1)
        if steps == 0:
            rows = torch.nonzero(keep).squeeze(1)
            active, features, legal, players = (t.index_select(0, rows)
                                                for t in (active, features, legal, players))
            started.index_fill_(0, active, True)
        else:
            bad += (~keep).sum()
        if active.numel() == 0:
            break
        seat = players.to(torch.int64)
        # Noise counter {deal seed, decision}: independent across games and iterations.
        dec = torch.full((active.numel(),), steps, dtype=torch.int32, device=device)
        actions, logp = _act_sample(ext, actor, features, legal, seeds.index_select(0, active), dec, 0)
        steps += 1
        opp_hand = ext.hands_indexed(states, active).gather(1, (1 - seat).unsqueeze(1)).squeeze(1)
        storage.append(features, legal, actions, logp, opp_hand, active, seat)
        reward0, new_done, nagari, step_status, _ = ext.step_indexed(states, active, actions)
        bad += (step_status != int(ext.STATUS_OK)).sum()
        final_reward0.index_copy_(0, active, torch.where(new_done, reward0, 0.0))
        final_nagari.index_copy_(0, active, new_done & nagari)
        active = active.index_select(0, torch.nonzero(~new_done).squeeze(1))
        if active.numel() == 0:
            break
    else:
        raise RuntimeError(f"games did not finish within {max_steps} steps")
    if int(bad):
        raise RuntimeError("an active game had no legal action, a bad status or a failed step")
    features, legal, actions, logp, opp_hand, env_ids, seat = storage.views()
    reward = final_reward0.index_select(0, env_ids)
    returns = torch.where(seat == 0, reward, -reward) / reward_scale
    return Rollout(features, legal, actions, logp, opp_hand, env_ids, seat, returns, games,
                   terminal=int((started & ~final_nagari).sum()),
                   nagari=int((started & final_nagari).sum()), decision_steps=steps,
                   mean_abs_reward0=float(final_reward0[started].abs().mean()))


def gae_advantages(values: torch.Tensor, returns: torch.Tensor, env_ids: torch.Tensor,
                   seat: torch.Tensor, lam: float) -> torch.Tensor:
    """GAE(lambda) with gamma 1 along each (game, seat) sequence of own decisions
    (python/cugo_ppo50.py:484-509): delta_t = V(next own decision) - V(t), the last
    decision's next value is the return; lam >= 1 gives return - V.  Rows are in
    step order within each game."""
    if lam >= 1.0:
        return returns - values
    n = values.numel()
    order = torch.sort(env_ids * 2 + seat, stable=True).indices
    key = (env_ids * 2 + seat).index_select(0, order)
    nxt_same = torch.zeros(n, dtype=torch.bool, device=values.device)
    nxt_same[:-1] = key[1:] == key[:-1]
    v = values.index_select(0, order)
    ret = returns.index_select(0, order)
    delta = torch.where(nxt_same, torch.roll(v, -1), ret) - v
    # Distance of each row to the end of its sequence.
    pos = torch.arange(n, device=values.device)
    end = torch.where(nxt_same, n, pos).flip(0).cummin(0).values.flip(0)
    dist = end - pos
    adv = torch.zeros_like(v)
    for d in range(int(dist.max()) + 1 if n else 0):
        rows = torch.nonzero(dist == d).squeeze(1)
        adv[rows] = delta[rows] + (lam * adv[rows + 1] if d else 0.0)
    out = torch.empty_like(adv)
    out[order] = adv
    return out


@dataclass
class TrainStats:
    """python/cugo_ppo50.py:460-476 (the plain-target fields)."""
    policy_loss: float
    value_loss: float
    entropy: float
    kl: float
    clipfrac: float
    explained_var: float
    updates: int
    epochs: float


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
                 grad_clip: float = 1.0, use_graph: bool = True, world: int = 1) -> None:
        self.actor, self.critic, self.minibatch = actor, critic, minibatch
        params = list(actor.parameters()) + list(critic.parameters())
        self.optimizer = torch.optim.Adam(params, lr=lr, capturable=use_graph)
        self.step = PpoStep(actor, critic, self.optimizer, clip, value_coef, grad_clip, world)
        self.use_graph = use_graph
        self.world = world
        self.graphed: GraphedPpoStep | None = None

    def _steps_per_epoch(self, n: int, device: torch.device) -> int:
        steps = n // self.minibatch
        if self.world > 1:
            t = torch.tensor([steps], dtype=torch.int64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            steps = int(t)
        return steps

    def _kl(self) -> float:
        kl = self.step.last_kl.detach().reshape(1).clone()
        if self.world > 1:
            dist.all_reduce(kl)
            kl /= self.world
        return float(kl)

    @torch.no_grad()
    def values(self, data: Rollout, chunk: int = 65536) -> torch.Tensor:
        self.critic.eval()
        n = data.actions.numel()
        return torch.cat([self.critic(critic_input(data.features[i:i + chunk],
                                                   data.opp_hand[i:i + chunk])).float().reshape(-1)
                          for i in range(0, n, chunk)]) if n else torch.zeros(0, device=data.returns.device)

    def update(self, data: Rollout, epochs: int, entropy_coef: float, target_kl: float,
               gae_lambda: float = 1.0) -> TrainStats:
        n = data.actions.numel()
        values = self.values(data)
        adv = gae_advantages(values, data.returns, data.env_ids, data.seat, gae_lambda)
        ret = adv + values
        explained_var = 1.0 - float((data.returns - values).var() /
                                    data.returns.var().clamp_min(1e-8))
        self.actor.train()
        self.critic.train()
        st = self.step
        st.entropy_coef.fill_(entropy_coef)
        st.sums.zero_()
        updates, stop = 0, False
        steps = self._steps_per_epoch(n, data.actions.device)
        for _ in range(epochs):
            perm = torch.randperm(n, device=data.actions.device)
            for j in range(steps):
                idx = perm[j * self.minibatch:(j + 1) * self.minibatch]
                mb = Minibatch(data.features.index_select(0, idx), data.legal.index_select(0, idx),
                               data.actions.index_select(0, idx), data.logp.index_select(0, idx),
                               data.opp_hand.index_select(0, idx), adv.index_select(0, idx),
                               ret.index_select(0, idx))
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
        s = st.sums.tolist()
        count = max(1.0, s[5])
        return TrainStats(policy_loss=s[0] / count, value_loss=s[1] / count, entropy=s[2] / count,
                          kl=s[3] / count, clipfrac=s[4] / count, explained_var=explained_var,
                          updates=updates, epochs=updates / max(1, steps))


def iteration(ext: Any, trainer: PpoTrainer, storage: RolloutStorage, games: int,
              seed_offset: int, reward_scale: float = 32.0, epochs: int = 2,
              entropy_coef: float = 0.05, target_kl: float = 0.03,
              gae_lambda: float = 0.95) -> dict:
    """One train_ppo50.py iteration (its defaults: 65,536 games, 2 epochs, minibatch
    32,768, GAE 0.95, reward scale 32): collection and update, timed on the host
    around device synchronisations.  Data parallel: each rank passes its own
    seed_offset (disjoint games) and a trainer built with world = the number of ranks."""
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    data = collect(ext, trainer.actor, games, seed_offset, reward_scale, storage)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    stats = trainer.update(data, epochs, entropy_coef, target_kl, gae_lambda)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    return dict(collect_seconds=t1 - t0, update_seconds=t2 - t1, seconds=t2 - t0,
                rows=int(data.actions.numel()), games=games, decision_steps=data.decision_steps,
                stats=stats)
