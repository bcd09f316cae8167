"""GPU: one PPO iteration (python/cugo_ppo50.py collect :321-450, update :514-745) on the
native kernels.  collect's transitions equal those of the collection loop restated
with the separate ops (observe, the actor's forward, the sampler with the same noise
counters, step); the update runs its epochs of graphed minibatch steps and moves both
networks."""
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


def _restated_collect(ext, actor, games, seed_offset, reward_scale):
    from cugo_b200.evaluate import make_seeds
    seeds, first = make_seeds(games, seed_offset, DEV)
    states = ext.create(seeds, first)
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
        with torch.no_grad():
            logits = actor(f).float().contiguous()
        dec = torch.full((active.numel(),), steps, dtype=torch.int32, device=DEV)
        a, lp = ext.sample_actions(logits, legal, seeds[active], dec, 0)
        steps += 1
        opp = ext.hands_indexed(states, active).gather(1, (1 - seat).unsqueeze(1)).squeeze(1)
        rows.append((f, legal, a, lp, opp, active.clone(), seat))
        r0, nd, _, _, _ = ext.step_indexed(states, active, a)
        final.index_copy_(0, active, torch.where(nd, r0, 0.0))
        active = active[~nd]
        if active.numel() == 0:
            break
    cols = [torch.cat(c) for c in zip(*rows)]
    reward = final[cols[5]]
    cols.append(torch.where(cols[6] == 0, reward, -reward) / reward_scale)
    return cols, steps


def test_collect_matches_the_separate_ops_loop(ext):
    from cugo_b200.train import RolloutStorage, collect
    actor, _ = _nets()
    data = collect(ext, actor, 3000, 17, 32.0, RolloutStorage(1000, DEV))
    cols, steps = _restated_collect(ext, actor, 3000, 17, 32.0)
    got = (data.features, data.legal, data.actions, data.opp_hand, data.env_ids, data.seat,
           data.returns)
    for a, b in zip(got, (cols[0], cols[1], cols[2], cols[4], cols[5], cols[6], cols[7])):
        assert torch.equal(a, b)
    assert float((data.logp - cols[3]).abs().max()) <= 1e-5
    assert data.decision_steps == steps
    assert bool(data.legal.gather(1, data.actions.unsqueeze(1)).all())


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
