"""GPU: all-action and redealt-world branching (python/cugo_ppo50.py:84-270) on the
native kernels.

- observe_critic_bf16 writes exactly [observe_indexed features, the hand plane of
  the mover's opponent, zero padding] (the reference builds it from observe_indexed,
  hands_indexed and card_plane, python/cugo_ppo50.py:97-101,478-482).
- cugo_b200_redeal is bit-exact with the numpy restatement of the redeal.
- redeal_worlds keeps the observer's view: features and legal actions of every
  world equal the real deal's, cards are conserved.
- action_values equals the reference's composition with the same critic bit for
  bit (fp16 results), for a scalar and a distributional value head.
- greedy_to_end equals greedy play on the oracle engine (bit-exact scores), with
  and without a pool opponent.
- world_values (depth 1) is the mean over the redealt worlds of action_values in
  each world, within fp16 rounding.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests import redeal_reference as rr

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SCALE = 10.0


def _roots(ext, n, seed):
    states = ext.branch_roots(n, seed_base=seed, device=DEV)
    ids = torch.arange(n, device=DEV)
    _, legal, players, done, _ = ext.observe_indexed(states, ids)
    keep = torch.nonzero(~done).squeeze(1)
    states = states.index_select(0, keep).contiguous()
    return states, legal.index_select(0, keep), players.index_select(0, keep).long()


def _critic(bins=0, seed=0):
    from cugo_b200.ppo import fused_critic
    torch.manual_seed(seed)
    c = fused_critic(hidden=256, blocks=2, value_bins=bins).to(DEV)
    with torch.no_grad():
        for p in c.parameters():
            p.copy_(torch.randn_like(p) * (1.0 / p.shape[-1]) ** 0.5)
    return c


def _plane(masks):
    bits = torch.arange(50, device=masks.device)
    return ((masks.view(-1, 1) >> bits) & 1).to(torch.bfloat16)


def test_observe_critic_rows(ext):
    states, _, _ = _roots(ext, 3000, 41)
    n = states.shape[0]
    g = torch.Generator(device="cpu").manual_seed(3)
    ids = torch.randint(0, n, (2 * n + 5,), generator=g).to(DEV)
    ids[7] = n + 4  # out of range: a zero row reported done with status -1
    crit, players, done, status = ext.observe_critic_bf16(states, ids)
    f, _, p2, d2, s2 = ext.observe_indexed_bf16(states, ids)
    assert torch.equal(players, p2) and torch.equal(done, d2) and torch.equal(status, s2)
    assert torch.equal(crit[:, :720], f)
    hands = ext.hands_indexed(states, ids)
    opp = hands.gather(1, (1 - players.long()).unsqueeze(1)).squeeze(1)
    opp[7] = 0
    assert torch.equal(crit[:, 720:770], _plane(opp))
    assert not crit[:, 770:].any()
    assert int(status[7]) == -1 and bool(done[7])


@pytest.mark.parametrize("seed,attempt", [(0, 0), (123456789, 3), (-5, 7)])
def test_redeal_matches_restatement(ext, seed, attempt):
    states, _, players = _roots(ext, 2048, 17 + attempt)
    rows = states.clone()
    ext.redeal(rows, players, seed, attempt)
    expect = rr.redeal(states.cpu().numpy(), players.cpu().numpy(), seed, attempt)
    assert np.array_equal(rows.cpu().numpy(), expect)


@pytest.mark.parametrize("worlds,tries,seed", [(3, 8, 9), (2, 1, -4), (4, 0, 1)])
def test_redeal_worlds_match_restatement(ext, oracle, worlds, tries, seed):
    states, _, players = _roots(ext, 700, 61)
    g = torch.Generator(device="cpu").manual_seed(worlds)
    env_rows = torch.randint(0, states.shape[0], (300,), generator=g).to(DEV)
    seats = players.index_select(0, env_rows)
    out, kept = ext.redeal_worlds(states, env_rows, seats, worlds, seed=seed, tries=tries,
                                  with_attempts=True)
    e_out, e_kept = rr.redeal_worlds(oracle, states.cpu().numpy(), env_rows.cpu().numpy(),
                                     seats.cpu().numpy(), worlds, seed, tries)
    assert np.array_equal(kept.cpu().numpy(), e_kept)
    assert np.array_equal(out.cpu().numpy(), e_out)
    if tries:
        assert (e_kept >= 0).mean() > 0.85


def test_redeal_worlds_keep_the_observer_view(ext):
    from cugo_b200.allaction import redeal_worlds
    states, _, players = _roots(ext, 1024, 5)
    r = states.shape[0]
    env_rows = torch.arange(r, device=DEV)
    worlds = redeal_worlds(ext, states, env_rows, players, 4, seed=9)
    assert worlds.shape == (4 * r, 248)
    ids = torch.arange(4 * r, device=DEV)
    f, l = ext.observe_indexed(worlds, ids)[:2]
    f0, l0 = ext.observe_indexed(states, env_rows)[:2]
    assert torch.equal(f, f0.repeat(4, 1)) and torch.equal(l, l0.repeat(4, 1))
    a = states.repeat(4, 1).view(torch.int64)
    b = worlds.view(torch.int64)
    seat = players.repeat(4)
    opp = torch.where(seat == 0, 1, 0)
    ar = torch.arange(4 * r, device=DEV)
    assert torch.equal(a[ar, opp] | a[:, 3], b[ar, opp] | b[:, 3])
    assert float((a[ar, opp] != b[ar, opp]).float().mean()) > 0.8  # most worlds differ


@pytest.mark.parametrize("bins", [0, 51])
def test_action_values_match_the_reference_composition(ext, bins):
    from cugo_b200.allaction import action_values
    from cugo_b200.ppo import critic_input
    states, legal, players = _roots(ext, 1500, 23)
    r = states.shape[0]
    g = torch.Generator(device="cpu").manual_seed(1)
    branch = legal & (torch.rand(legal.shape, generator=g) < 0.7).to(DEV)
    env_rows = torch.arange(r, device=DEV)
    critic = _critic(bins)
    q = action_values(ext, critic, states, env_rows, players, branch, SCALE)
    # The reference's steps (python/cugo_ppo50.py:91-104) with the same critic.
    rows, acts = torch.nonzero(branch, as_tuple=True)
    m = players.index_select(0, rows)
    child, reward0, done = ext.branch_indexed(states, rows, acts)[:3]
    ids = torch.arange(child.shape[0], device=DEV)
    features, _, mover, _, _ = ext.observe_indexed(child, ids)
    mover = mover.long()
    opp = ext.hands_indexed(child, ids).gather(1, (1 - mover).unsqueeze(1)).squeeze(1)
    with torch.no_grad():
        v = critic.value(critic(critic_input(features, opp)))
    v = torch.where(mover == m, v, -v)
    final = torch.where(m == 0, reward0, -reward0) / SCALE
    expect = torch.full(branch.shape, float("nan"), dtype=torch.float16, device=DEV)
    expect[rows, acts] = torch.where(done, final, v).to(torch.float16)
    assert torch.equal(torch.isnan(q), ~branch)
    assert torch.equal(q[branch], expect[branch])
    assert bool(done.any()) and bool((~done).any())


def _oracle_greedy(oracle, child, done, me, pool):
    """Greedy play to the end on the oracle engine: the learner (and every seat of a
    non-pool game) takes its lowest legal action, the pool opponent its highest."""
    rows = child.copy()
    final = np.zeros(rows.shape[0], dtype=np.float32)
    running = ~done.copy()
    for _ in range(96):
        if not running.any():
            break
        idx = np.nonzero(running)[0]
        _, legal, player, _, _ = oracle.observe(rows[idx], threads=1)
        low = legal.argmax(1)
        high = legal.shape[1] - 1 - legal[:, ::-1].argmax(1)
        theirs = pool[idx] & (player.astype(np.int64) != me[idx])
        act = np.where(theirs, high, low)
        new, reward, nd = oracle.step(rows[idx], act, threads=1)[:3]
        rows[idx] = new
        final[idx] = reward
        running[idx] = ~nd
    assert not running.any()
    return final


@pytest.mark.parametrize("with_pool", [False, True])
def test_greedy_to_end_matches_the_oracle(ext, oracle, with_pool):
    from cugo_b200.allaction import greedy_to_end
    from cugo_b200.ppo import fused_actor
    states, legal, players = _roots(ext, 600, 31)
    rows, acts = torch.nonzero(legal, as_tuple=True)
    child, reward0, done = ext.branch_indexed(states, rows, acts)[:3]
    me = players.index_select(0, rows)
    g = torch.Generator(device="cpu").manual_seed(2)
    pool = (torch.rand(rows.numel(), generator=g) < 0.5).to(DEV)
    actor = fused_actor(hidden=256, blocks=2).to(DEV)  # zero output: lowest legal action
    opponent = None
    if with_pool:
        opponent = fused_actor(hidden=256, blocks=2).to(DEV)
        with torch.no_grad():  # logits = action index: highest legal action
            opponent.out.bias.copy_(torch.arange(179, dtype=torch.float32))
    child_np = child.cpu().numpy()
    final = greedy_to_end(ext, actor, opponent, child, reward0, done, me, pool)
    expect = _oracle_greedy(oracle, child_np, done.cpu().numpy(), me.cpu().numpy(),
                            pool.cpu().numpy() & with_pool)
    expect = np.where(done.cpu().numpy(), reward0.cpu().numpy(), expect)
    assert np.array_equal(final.cpu().numpy(), expect)


def test_world_values_average_the_worlds(ext):
    from cugo_b200.allaction import action_values, redeal_worlds, world_values
    states, legal, players = _roots(ext, 400, 77)
    r = states.shape[0]
    env_rows = torch.arange(r, device=DEV)
    critic = _critic(0, seed=4)
    vs_pool = torch.zeros(r, dtype=torch.bool, device=DEV)
    q = world_values(ext, None, None, states, env_rows, players, vs_pool, legal, SCALE, 3,
                     critic=critic, depth=1, seed=21)
    worlds = redeal_worlds(ext, states, env_rows, players, 3, seed=21)
    per = [action_values(ext, critic, worlds, env_rows + k * r, players, legal, SCALE).float()
           for k in range(3)]
    expect = torch.stack(per).mean(0)
    assert torch.equal(torch.isnan(q), ~legal)
    assert torch.allclose(q[legal].float(), expect[legal], rtol=2e-3, atol=2e-3)
    # first < worlds: two worlds first, the third only where their best actions differ.
    q2 = world_values(ext, None, None, states, env_rows, players, vs_pool, legal, SCALE, 3,
                      critic=critic, depth=1, first=2, seed=21)
    assert torch.equal(torch.isnan(q2), ~legal) and bool(torch.isfinite(q2[legal]).all())


def test_action_values_with_a_stock_critic(ext):
    """OracleCritic(stock=True) (python/cugo_ppo_nets50.py:67-87): the critic rows get the
    one-hot planes of the next 8 stock draws in the observe pass (observe_critic_bf16
    then stock_planes_bf16), equal to the reference's composition with stock_indexed."""
    from cugo_b200.allaction import action_values
    from cugo_b200.ppo import critic_input, fused_critic
    states, legal, players = _roots(ext, 1200, 29)
    r = states.shape[0]
    torch.manual_seed(8)
    critic = fused_critic(hidden=256, blocks=2, stock=True).to(DEV)
    with torch.no_grad():
        for p in critic.parameters():
            p.copy_(torch.randn_like(p) * (1.0 / p.shape[-1]) ** 0.5)
    env_rows = torch.arange(r, device=DEV)
    q = action_values(ext, critic, states, env_rows, players, legal, SCALE)
    rows, acts = torch.nonzero(legal, as_tuple=True)
    m = players.index_select(0, rows)
    child, reward0, done = ext.branch_indexed(states, rows, acts)[:3]
    ids = torch.arange(child.shape[0], device=DEV)
    features, _, mover, _, _ = ext.observe_indexed(child, ids)
    mover = mover.long()
    opp = ext.hands_indexed(child, ids).gather(1, (1 - mover).unsqueeze(1)).squeeze(1)
    stock = ext.stock_indexed(child, ids)
    crit_rows, _, _, _ = ext.observe_critic_bf16(child, ids, width=1176)
    ext.stock_planes_bf16(child, ids, crit_rows)
    assert torch.equal(crit_rows[:, :1170], critic_input(features, opp, stock))
    assert not crit_rows[:, 1170:].any()
    with torch.no_grad():
        v = critic.value(critic(critic_input(features, opp, stock)))
    v = torch.where(mover == m, v, -v)
    final = torch.where(m == 0, reward0, -reward0) / SCALE
    expect = torch.where(done, final, v).to(torch.float16)
    assert torch.equal(q[rows, acts], expect)
