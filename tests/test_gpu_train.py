"""GPU: one PPO iteration (python/cugo_ppo50.py collect :321-450, update :514-745) on the
native kernels.  collect's transitions (the device-resident store written by the record
kernel) equal those of the collection loop restated with the separate ops (observe, the
actor's forward, the sampler with the same noise counters, hands, stock preview, step),
with and without a pool opponent; the update runs its epochs of graphed minibatch steps
and moves both networks, also with a critic that reads the stock planes."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _nets():
    from cugo_b200.ppo import fused_actor, fused_critic
    torch.manual_seed(0)
    actor, critic = fused_actor().to(DEV), fused_critic().to(DEV)
    with torch.no_grad():  # a non-trivial actor (the real one starts at zero logits)
        actor.out.weight.normal_(0.0, 0.02)
    return actor, critic


def _restated_collect(ext, actor, games, seed_offset, reward_scale, pool=None, pool_fraction=0.0,
                      pool_greedy=False):
    """The collection loop with separate ops: observe, the actor's forward and the
    sampler (noise counter {deal seed, decision}), the pool opponent where it moves
    (seed base 1), step, and the learner's transitions kept in round order."""
    from cugo_b200.evaluate import make_seeds
    seeds, first = make_seeds(games, seed_offset, DEV)
    states = ext.create(seeds, first)
    opponent = pool[int(torch.randint(len(pool), ()))] if pool and pool_fraction > 0 else None
    learner_seat = torch.randint(2, (games,), device=DEV)
    vs_pool = torch.rand(games, device=DEV) < pool_fraction if opponent is not None else None
    active = torch.arange(games, device=DEV)
    final = torch.zeros(games, device=DEV)
    rows = []
    steps = 0
    while True:
        f, legal, players, done, status = ext.observe_indexed_bf16(states, active)
        if steps == 0:
            keep = torch.nonzero(~done & (status == 0) & legal.any(1)).squeeze(1)
            active, f, legal, players = active[keep], f[keep], legal[keep], players[keep]
        seat = players.long()
        dec = torch.full((active.numel(),), steps, dtype=torch.int32, device=DEV)
        with torch.no_grad():
            a, lp = ext.sample_actions(actor(f).float().contiguous(), legal, seeds[active], dec, 0)
            mine = torch.ones_like(a, dtype=torch.bool)
            if opponent is not None:
                theirs = ext.sample_actions(opponent(f).float().contiguous(), legal, seeds[active],
                                            dec, 1, greedy=pool_greedy)[0]
                mine = ~vs_pool[active] | (seat == learner_seat[active])
                a = torch.where(mine, a, theirs)
        steps += 1
        opp = ext.hands_indexed(states, active).gather(1, (1 - seat).unsqueeze(1)).squeeze(1)
        stock = ext.stock_indexed(states, active)
        k = mine
        rows.append((f[k], legal[k], a[k], lp[k], opp[k], active[k].clone(), seat[k], stock[k]))
        r0, nd, _, _, _ = ext.step_indexed(states, active, a)
        final.index_copy_(0, active, torch.where(nd, r0, 0.0))
        active = active[~nd]
        if active.numel() == 0:
            break
    cols = [torch.cat(c) for c in zip(*rows)]
    reward = final[cols[5]]
    cols.append(torch.where(cols[6] == 0, reward, -reward) / reward_scale)
    return cols, steps


def _check_rollout(data, cols, steps):
    got = (data.features, data.legal, data.actions, data.opp_hand, data.env_ids, data.seat,
           data.stock, data.returns)
    names = ("features", "legal", "actions", "opp_hand", "env_ids", "seat", "stock", "returns")
    for name, a, b in zip(names, got, (cols[0], cols[1], cols[2], cols[4], cols[5], cols[6],
                                       cols[7], cols[8])):
        assert a.shape == b.shape and torch.equal(a, b), name
    assert float((data.logp - cols[3]).abs().max()) <= 1e-5
    assert data.decision_steps == steps
    assert bool(data.legal.gather(1, data.actions.unsqueeze(1)).all())


def test_collect_matches_the_separate_ops_loop(ext):
    """A fused actor: no host read per round; a store of 1,000 rows grows on the way."""
    from cugo_b200.train import RolloutStorage, collect
    actor, _ = _nets()
    storage = RolloutStorage(1000, DEV)
    data = collect(ext, actor, [], 3000, 17, 0.0, False, 32.0, storage)
    assert storage.capacity > 1000
    cols, steps = _restated_collect(ext, actor, 3000, 17, 32.0)
    _check_rollout(data, cols, steps)


@pytest.mark.parametrize("greedy,hidden", [(False, 512), (True, 256)])
def test_collect_with_a_pool_opponent(ext, greedy, hidden):
    """Pool games (half of them): the opponent moves where it is to play and only the
    learner's decisions are kept; a 256-wide opponent takes the generic path."""
    from cugo_b200.ppo import fused_actor
    from cugo_b200.train import RolloutStorage, collect
    actor, _ = _nets()
    torch.manual_seed(3)
    opp = fused_actor(hidden=hidden).to(DEV)
    with torch.no_grad():
        opp.out.weight.normal_(0.0, 0.05)
    torch.manual_seed(11)
    data = collect(ext, actor, [opp], 2500, 23, 0.5, greedy, 32.0, RolloutStorage(70000, DEV))
    torch.manual_seed(11)
    cols, steps = _restated_collect(ext, actor, 2500, 23, 32.0, [opp], 0.5, greedy)
    _check_rollout(data, cols, steps)
    assert data.learner_score == data.learner_score  # pool games were played


def test_iteration_updates_both_networks(ext):
    from cugo_b200.train import PpoTrainer, RolloutStorage, iteration
    actor, critic = _nets()
    before = [p.detach().clone() for p in list(actor.parameters()) + list(critic.parameters())]
    trainer = PpoTrainer(actor, critic, minibatch=4096)
    out = iteration(ext, trainer, RolloutStorage(1 << 16, DEV), 2048, 5, epochs=2, target_kl=0.0)
    st = out["stats"]
    assert out["rows"] > 2048 * 5 and st.updates == 2 * (out["rows"] // 4096)
    for v in (st.policy_loss, st.value_loss, st.entropy, st.kl, st.clipfrac, st.explained_var):
        assert v == v and abs(v) < 1e6  # finite
    after = list(actor.parameters()) + list(critic.parameters())
    assert all(not torch.equal(a, b) for a, b in zip(before, after) if a.numel() > 1)


def test_iteration_with_a_stock_critic(ext):
    from cugo_b200.ppo import fused_critic
    from cugo_b200.train import PpoTrainer, RolloutStorage, iteration
    actor, _ = _nets()
    critic = fused_critic(hidden=256, blocks=2, stock=True).to(DEV)
    assert critic.inp.in_features == 1170
    before = critic.inp.weight.detach().clone()
    trainer = PpoTrainer(actor, critic, minibatch=4096)
    out = iteration(ext, trainer, RolloutStorage(1 << 16, DEV), 2048, 9, epochs=1, target_kl=0.0)
    assert out["stats"].updates >= 1
    assert not torch.equal(before, critic.inp.weight)
