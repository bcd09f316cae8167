"""Restatement of the reference's paired evaluator loop (TEST INFRASTRUCTURE ONLY).

python/cugo_eval50.py:137-361: host-side compaction of the running games every
decision step, each policy applied to its own rows, greedy masked argmax, the same
statistics.  Run here with the extension's ops and the same policy modules as the
fused evaluator, so both must agree exactly.
"""
from __future__ import annotations

import math

import torch

SIGNED_GOLDEN = -7046029254386353131
SEED_BASE = 0x243F6A8885A308D3


def _greedy(model, features, legal):
    out = model(features)
    logits = (out[0] if isinstance(out, tuple) else out).float()
    return logits.masked_fill(~legal, -1.0e30).argmax(dim=1).to(torch.int64)


@torch.no_grad()
def evaluate_paired(ext, model_a, model_b, pairs: int, seed_offset: int, max_steps: int) -> dict:
    device = torch.device("cuda")
    index = torch.arange(pairs, dtype=torch.int64, device=device)
    base_seeds = index.mul(SIGNED_GOLDEN).add(SEED_BASE + seed_offset)
    base_first = index.bitwise_and(1)
    seeds, first = torch.cat((base_seeds, base_seeds)), torch.cat((base_first, base_first))
    games = 2 * pairs
    a_seat = torch.cat((torch.zeros(pairs, dtype=torch.uint8, device=device),
                        torch.ones(pairs, dtype=torch.uint8, device=device)))
    states = ext.create(seeds, first)
    final_reward0 = torch.zeros(games, device=device)
    final_nagari = torch.zeros(games, dtype=torch.bool, device=device)
    predecision_done = torch.zeros(games, dtype=torch.bool, device=device)
    active_ids = torch.arange(games, dtype=torch.int64, device=device)
    bad = [0, 0, 0]
    completed, first_observe, decision_steps = False, True, 0
    for _ in range(max_steps):
        if active_ids.numel() == 0:
            completed = True
            break
        features, legal, players, observed_done, status = ext.observe_indexed(states, active_ids)
        ok = status == 0
        has_legal = legal.any(dim=1)
        if first_observe:
            active = ~observed_done
            valid = active & ok & has_legal
            done_rows = torch.nonzero(observed_done).squeeze(1)
            if done_rows.numel():
                predecision_done.index_fill_(0, active_ids.index_select(0, done_rows), True)
            bad[0] += int((active & ~ok).sum())
            bad[1] += int((active & ok & ~has_legal).sum())
            keep = torch.nonzero(valid).squeeze(1)
            active_ids = active_ids.index_select(0, keep)
            features, legal = features.index_select(0, keep), legal.index_select(0, keep)
            players = players.index_select(0, keep)
            first_observe = False
            if active_ids.numel() == 0:
                completed = True
                break
        else:
            bad[0] += int((~ok).sum())
            bad[1] += int((ok & (observed_done | ~has_legal)).sum())
        decision_steps += 1
        use_a = players.to(torch.int64) == a_seat.index_select(0, active_ids).to(torch.int64)
        a_rows = torch.nonzero(use_a).squeeze(1)
        b_rows = torch.nonzero(~use_a).squeeze(1)
        actions = torch.empty(active_ids.numel(), dtype=torch.int64, device=device)
        if a_rows.numel():
            actions.index_copy_(0, a_rows, _greedy(model_a, features.index_select(0, a_rows),
                                                   legal.index_select(0, a_rows)))
        if b_rows.numel():
            actions.index_copy_(0, b_rows, _greedy(model_b, features.index_select(0, b_rows),
                                                   legal.index_select(0, b_rows)))
        reward0, new_done, nagari, step_status, _ = ext.step_indexed(states, active_ids, actions)
        step_ok = step_status == 0
        bad[2] += int((~step_ok).sum())
        just = step_ok & new_done
        final_reward0.index_copy_(0, active_ids, torch.where(just, reward0, torch.zeros_like(reward0)))
        final_nagari.index_copy_(0, active_ids, just & nagari)
        active_ids = active_ids.index_select(0, torch.nonzero(step_ok & ~new_done).squeeze(1))
        if active_ids.numel() == 0:
            completed = True
            break
    assert completed and bad == [0, 0, 0]
    score_a = torch.where(a_seat == 0, final_reward0, -final_reward0)
    p0, p1 = score_a[:pairs], score_a[pairs:]
    pair = (p0 + p1) * 0.5

    def wdl(x):
        return int((x > 0).sum()), int((x < 0).sum()), int((x == 0).sum())

    p0_valid, p1_valid = ~predecision_done[:pairs], ~predecision_done[pairs:]
    pv = p0_valid & p1_valid
    valid = score_a[~predecision_done]
    vp = pair[pv]
    n_pairs = int(pv.sum())
    std = float(vp.std(unbiased=True)) if n_pairs > 1 else 0.0
    mean_pair = float(vp.mean()) if n_pairs else 0.0
    se = std / math.sqrt(n_pairs) if n_pairs > 1 else 0.0
    a_wins, b_wins, draws = wdl(valid)
    return dict(
        pairs=pairs, games=games, evaluated_pairs=n_pairs,
        evaluated_games=int((~predecision_done).sum()),
        predecision_excluded=int(predecision_done.sum()), a_wins=a_wins, b_wins=b_wins,
        draws=draws, a_p0=wdl(p0[p0_valid]), a_p1=wdl(p1[p1_valid]), pair=wdl(vp),
        mean_score_a=float(valid.mean()), mean_pair_score_a=mean_pair, pair_score_std=std,
        pair_score_ci95_low=mean_pair - 1.959963984540054 * se,
        terminal=int((~final_nagari).sum()), nagari=int(final_nagari.sum()),
        decision_steps=decision_steps, final_reward0=final_reward0)
