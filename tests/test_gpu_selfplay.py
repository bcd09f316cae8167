"""GPU: the self-play round on the fused kernels.

step_compact (the step kernel with a round's bookkeeping) against step_indexed plus
the same bookkeeping in torch; play_batch (observe with bit-word masks, the fused
policy-and-sampling kernel, step_compact) against the collection loop restated with
the separate ops (observe_indexed_bf16, policy forward, sample_actions, step_indexed,
torch compaction): the same final rewards, nagari flags, decision and round counts.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_step_compact_matches_step_indexed(ext):
    n = 6000
    idx = torch.arange(n, device=DEV, dtype=torch.int64)
    states = ext.create(idx + 4242, idx & 1)
    g = torch.Generator().manual_seed(9)
    for _ in range(12):  # advance with random legal actions; some games finish
        _, legal, _, _, _ = ext.observe_indexed(states, idx)
        logits = torch.randn((n, 180), generator=g).to(DEV)
        acts, _ = ext.sample_actions(logits, legal, idx, torch.zeros(n, dtype=torch.int32, device=DEV))
        ext.step_indexed(states, idx, acts.clamp_min(0))
    ids = torch.randperm(n, generator=g)[:4000].to(DEV)
    _, legal, _, _, _ = ext.observe_indexed(states, ids)
    logits = torch.randn((ids.numel(), 180), generator=g).to(DEV)
    acts, _ = ext.sample_actions(logits, legal, ids, torch.zeros(ids.numel(), dtype=torch.int32, device=DEV))
    acts[::97] = 178  # mostly illegal: counted as bad, state unchanged
    ref_states = states.clone()
    reward, done, nagari, status, _ = ext.step_indexed(ref_states, ids, acts)
    dec0 = torch.randint(0, 5, (n,), generator=g, dtype=torch.int32).to(DEV)
    decision, reward0, nag = dec0.clone(), torch.zeros(n, device=DEV), torch.zeros(n, dtype=torch.bool, device=DEV)
    bad = torch.zeros(1, dtype=torch.int64, device=DEV)
    nxt = torch.full((n,), -7, dtype=torch.int64, device=DEV)
    count = torch.zeros(1, dtype=torch.int32, device=DEV)
    ext.step_compact(states, ids, acts, decision, reward0, nag, bad, nxt, count)
    assert torch.equal(states, ref_states)
    exp_dec = dec0.clone()
    exp_dec[ids] += 1
    assert torch.equal(decision, exp_dec)
    exp_r, exp_n = torch.zeros(n, device=DEV), torch.zeros(n, dtype=torch.bool, device=DEV)
    exp_r[ids] = torch.where(done, reward, 0.0)
    exp_n[ids] = done & nagari
    assert torch.equal(reward0, exp_r) and torch.equal(nag, exp_n)
    assert int(bad) == int(((status != 0) & (status != 9)).sum()) > 0
    live = int(count)
    assert torch.equal(nxt[:live], ids[~done])  # in order
    assert bool(done.any()) and bool((status == 9).any())


def test_step_compact_grouped_orders_by_next_decision(ext):
    """The grouped round tail writes the same running games as the in-order one,
    grouped by their next decision -- primary plays, then pending floor choices,
    then prompts (Go/Stop, Gukjin, Chongtong) -- each group in env_ids order, with the
    same rows, decision counters, rewards, nagari flags and bad count."""
    n = 20000
    idx = torch.arange(n, device=DEV, dtype=torch.int64)
    states = ext.create(idx + 777, idx & 1)
    g = torch.Generator().manual_seed(21)
    for _ in range(10):
        _, legal, _, _, _ = ext.observe_indexed(states, idx)
        logits = torch.randn((n, 180), generator=g).to(DEV)
        acts, _ = ext.sample_actions(logits, legal, idx, torch.zeros(n, dtype=torch.int32, device=DEV))
        ext.step_indexed(states, idx, acts.clamp_min(0))
    ids = torch.randperm(n, generator=g)[:15000].to(DEV)
    _, legal, _, _, _ = ext.observe_indexed(states, ids)
    logits = torch.randn((ids.numel(), 180), generator=g).to(DEV)
    acts, _ = ext.sample_actions(logits, legal, ids, torch.zeros(ids.numel(), dtype=torch.int32, device=DEV))
    outs = []
    for grouped in (False, True):
        st = states.clone()
        decision = torch.zeros(n, dtype=torch.int32, device=DEV)
        reward0, nag = torch.zeros(n, device=DEV), torch.zeros(n, dtype=torch.bool, device=DEV)
        bad = torch.zeros(1, dtype=torch.int64, device=DEV)
        nxt = torch.full((n,), -7, dtype=torch.int64, device=DEV)
        count = torch.zeros(1, dtype=torch.int32, device=DEV)
        ext.step_compact(st, ids, acts, decision, reward0, nag, bad, nxt, count, grouped=grouped)
        outs.append((st, decision, reward0, nag, bad, nxt[:int(count)].clone()))
    (s0, d0, r0, n0, b0, order), (s1, d1, r1, n1, b1, grouped_ids) = outs
    for a, b in ((s0, s1), (d0, d1), (r0, r1), (n0, n1), (b0, b1)):
        assert torch.equal(a, b)
    # The next decision of each running game, from its legal actions: a floor choice
    # offers actions 127..176 only, a prompt 123..126 (Go/Stop, Chongtong) or 177..178
    # (Gukjin) only, a primary play actions below 123 (or none).
    _, legal, _, _, _ = ext.observe_indexed(s1, order)
    choice = legal[:, 127:177].any(1)
    prompt = legal[:, 123:127].any(1) | legal[:, 177:179].any(1)
    group = torch.where(choice, 1, torch.where(prompt, 2, 0))
    expect = torch.cat([order[group == q] for q in range(3)])
    assert int(count) > 0 and bool((group == 1).any()) and bool((group == 2).any())
    assert torch.equal(grouped_ids, expect)


@pytest.mark.parametrize("device_rows", [None, 100_003])
def test_step_compact_grouped_at_scale(ext, device_rows):
    """Round tails of 131,072 entries (the scan moves each thread's words as 16-byte
    vectors from about 100k entries on), with all of them stepped or only the first
    `device_rows` (a device-resident count, so the last vector reaches past the rows):
    the running games, grouped by next decision, as stepping those entries with
    step_indexed and grouping them from their legal actions gives."""
    n, m = 140_000, 131_072
    idx = torch.arange(n, device=DEV, dtype=torch.int64)
    states = ext.create(idx + 99, idx & 1)
    g = torch.Generator().manual_seed(5)
    for _ in range(8):
        _, legal, _, _, _ = ext.observe_indexed(states, idx)
        logits = torch.randn((n, 180), generator=g).to(DEV)
        acts, _ = ext.sample_actions(logits, legal, idx, torch.zeros(n, dtype=torch.int32, device=DEV))
        ext.step_indexed(states, idx, acts.clamp_min(0))
    ids = torch.randperm(n, generator=g)[:m].to(DEV)
    _, legal, _, _, _ = ext.observe_indexed(states, ids)
    logits = torch.randn((m, 180), generator=g).to(DEV)
    acts, _ = ext.sample_actions(logits, legal, ids, torch.zeros(m, dtype=torch.int32, device=DEV))
    k = m if device_rows is None else device_rows
    ref = states.clone()
    _, done, _, _, _ = ext.step_indexed(ref, ids[:k], acts[:k])
    order = ids[:k][~done]
    _, legal, _, _, _ = ext.observe_indexed(ref, order)
    choice = legal[:, 127:177].any(1)
    prompt = legal[:, 123:127].any(1) | legal[:, 177:179].any(1)
    group = torch.where(choice, 1, torch.where(prompt, 2, 0))
    expect = torch.cat([order[group == q] for q in range(3)])
    decision = torch.zeros(n, dtype=torch.int32, device=DEV)
    reward0, nag = torch.zeros(n, device=DEV), torch.zeros(n, dtype=torch.bool, device=DEV)
    bad = torch.zeros(1, dtype=torch.int64, device=DEV)
    nxt = torch.full((n,), -7, dtype=torch.int64, device=DEV)
    count = torch.zeros(1, dtype=torch.int32, device=DEV)
    m_dev = None if device_rows is None else torch.tensor([k], dtype=torch.int32, device=DEV)
    ext.step_compact(states, ids, acts, decision, reward0, nag, bad, nxt, count, m_dev=m_dev,
                     grouped=True)
    assert torch.equal(states, ref)
    assert int(count) == expect.numel() > 0
    assert torch.equal(nxt[:int(count)], expect)


def _reference_loop(ext, policy, game_index, seed_base=12345, max_rounds=128):
    """The collection loop with separate ops and torch bookkeeping; games that the
    deal ended take no decision (reward 0)."""
    g = game_index.numel()
    states = ext.create(game_index + seed_base, game_index & 1)
    decision = torch.zeros(g, dtype=torch.int32, device=DEV)
    reward0 = torch.zeros(g, device=DEV)
    nagari = torch.zeros(g, dtype=torch.bool, device=DEV)
    active = torch.nonzero(states[:, 239] == 0).squeeze(1)
    decisions = rounds = 0
    for rounds in range(1, max_rounds + 1):
        features, legal, _, _, _ = ext.observe_indexed_bf16(states, active)
        actions, _ = ext.sample_actions(policy.forward(features), legal,
                                        game_index.index_select(0, active),
                                        decision.index_select(0, active), seed_base)
        reward, new_done, new_nagari, status, _ = ext.step_indexed(states, active, actions)
        assert not bool((status != 0).any())
        decisions += active.numel()
        decision.index_add_(0, active, torch.ones_like(active, dtype=torch.int32))
        reward0.index_copy_(0, active, torch.where(new_done, reward, 0.0))
        nagari.index_copy_(0, active, new_done & new_nagari)
        active = active.index_select(0, torch.nonzero(~new_done).squeeze(1))
        if active.numel() == 0:
            break
    return reward0, nagari, decisions, rounds


@pytest.mark.parametrize("activation", ["relu", "silu"])
def test_play_batch_matches_the_separate_ops_loop(ext, activation):
    from cugo_b200.policy import ResidualMlpPolicy
    from cugo_b200.selfplay import play_batch
    pol = ResidualMlpPolicy(512, 3, activation, device=DEV, seed=5)
    assert pol.samples_in_kernel()
    games = torch.arange(100000, 104096, device=DEV)
    res = play_batch(ext, pol, games)
    r0, nag, decisions, rounds = _reference_loop(ext, pol, games)
    assert res.bad_status == 0
    assert res.decisions == decisions and res.rounds == rounds
    # The reference loop's forward runs the same fused kernel, so its logits, and with
    # them every sampled action, are identical.
    assert torch.equal(res.nagari, nag) and torch.equal(res.reward0, r0)


def test_device_count_loop_equals_the_synchronised_loop(ext):
    """The same batch with the running count read back every round (the timer's path)
    and every CHECK_EVERY rounds (kernels reading the count from device memory)."""
    from cugo_b200.policy import ResidualMlpPolicy
    from cugo_b200.selfplay import RoundTimer, play_batch
    pol = ResidualMlpPolicy(512, 3, "relu", device=DEV, seed=6)
    games = torch.arange(7000, device=DEV)
    timer = RoundTimer(enabled=True)
    a = play_batch(ext, pol, games, timer=timer)
    b = play_batch(ext, pol, games)
    assert (a.decisions, a.rounds, a.bad_status) == (b.decisions, b.rounds, b.bad_status)
    assert torch.equal(a.reward0, b.reward0) and torch.equal(a.nagari, b.nagari)
    assert timer.total_ms()[2] == a.decisions  # the timer saw every round's rows


@pytest.mark.parametrize("games_from", [0, 500000])
def test_play_batch_replays_on_the_oracle(ext, oracle, games_from):
    """play_batch's recorded actions, replayed game by game on the reference's own
    engine (oracle/_ref): identical final rewards, nagari flags and decision counts,
    and no bad status on either side."""
    import numpy as np

    from cugo_b200.policy import ResidualMlpPolicy
    from cugo_b200.selfplay import play_batch
    from tests.replay import replay_on_oracle
    pol = ResidualMlpPolicy(512, 3, "relu", device=DEV, seed=0)
    g = 8192
    games = torch.arange(games_from, games_from + g, device=DEV)
    log = torch.full((g + 1, 64), -1, dtype=torch.int64, device=DEV)
    res = play_batch(ext, pol, games, actions_log=log)
    assert res.bad_status == 0
    per_game = int((log[:g] >= 0).sum())
    assert per_game == res.decisions
    r0, nag, dec, bad = replay_on_oracle(oracle, games.cpu().numpy(), log[:g].cpu().numpy())
    assert bad == 0
    assert int(dec.sum()) == res.decisions
    assert np.array_equal(r0, res.reward0.cpu().numpy())
    assert np.array_equal(nag, res.nagari.cpu().numpy())


def test_create_indexed_matches_create(ext):
    idx = torch.randint(0, 1 << 40, (5000,), device=DEV, dtype=torch.int64)
    a = ext.create_indexed(idx, 777)
    b = ext.create(idx + 777, idx & 1)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ext.create_indexed(idx[:0], 777).shape == (0, ext.STATE_BYTES)


@pytest.mark.parametrize("n", [0, 1, 31, 4097])
def test_running_init_lists_the_games_the_deal_left_running(ext, n):
    idx = torch.arange(n, device=DEV, dtype=torch.int64)
    states = ext.create_indexed(idx, 12345)
    if n:  # end some games at the deal by hand: their done byte is set
        ended = torch.rand(n, device=DEV) < 0.3
        states[ended, 239] = 1
    running = states[:, 239] == 0
    ids = torch.full((n + 5,), -7, dtype=torch.int64, device=DEV)
    count = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    decision = torch.full((n,), 9, dtype=torch.int32, device=DEV)
    reward0 = torch.full((n,), 3.0, device=DEV)
    nagari = torch.ones(n, dtype=torch.bool, device=DEV)
    bad = torch.full((1,), 5, dtype=torch.int64, device=DEV)
    scratch = torch.empty(max(1, 2 * ((n + 31) // 32)), dtype=torch.int32, device=DEV)
    spare = torch.full((n,), -7, dtype=torch.int64, device=DEV)
    ext.running_init(states, ids, count, decision, reward0, nagari, bad, scratch, spare_ids=spare)
    torch.cuda.synchronize()
    k = int(count)
    assert k == int(running.sum())
    assert torch.equal(ids[:k], torch.nonzero(running).squeeze(1))
    pos = torch.arange(n, device=DEV)
    assert torch.equal(ids[k:n], pos[k:]) and torch.equal(spare, pos)  # valid rows everywhere
    assert bool((ids[n:] == -7).all())  # nothing past n written
    assert not decision.any() and not reward0.any() and not nagari.any() and int(bad) == 0
