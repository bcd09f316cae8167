"""CPU: the host arithmetic of the paired evaluator (python/league50.py:25-28,
python/cugo_ppo_nets50.py:15-17, python/cugo_eval50.py:281-361)."""
from __future__ import annotations

import math

import torch

from cugo_b200.evaluate import chunk_offset, make_seeds, summarize


def test_chunk_offset_continues_the_deal_sequence():
    cpu = torch.device("cpu")
    for offset in (910000000, 0, -12345, 2 ** 62):
        seeds, first = make_seeds(1000, offset, cpu)
        for start in (0, 2, 400, 998):
            s, f = make_seeds(2, chunk_offset(offset, start), cpu)
            assert int(s[0]) == int(seeds[start]) and int(s[1]) == int(seeds[start + 1])
            assert int(f[0]) == int(first[start]) % 2 or start % 2 == 0


def test_summary_statistics():
    pairs = 4
    reward0 = torch.tensor([3.0, -2.0, 0.0, 5.0, 3.0, 1.0, 0.0, -5.0])
    nagari = torch.tensor([False, False, True, False, False, False, True, False])
    pre = torch.tensor([False, False, False, True, False, False, False, False])
    a_seat = torch.tensor([0, 0, 0, 0, 1, 1, 1, 1])
    s = summarize(reward0, nagari, pre, a_seat, pairs, 17, 2.0)
    score = [3.0, -2.0, 0.0, 5.0, -3.0, -1.0, -0.0, 5.0]
    valid = [x for i, x in enumerate(score) if i != 3]
    assert (s.a_wins, s.b_wins, s.draws) == (2, 3, 2)
    assert s.evaluated_games == 7 and s.evaluated_pairs == 3 and s.predecision_excluded == 1
    pair = [(score[i] + score[i + 4]) / 2 for i in range(3)]
    assert abs(s.mean_pair_score_a - sum(pair) / 3) < 1e-6
    mean = sum(pair) / 3
    std = math.sqrt(sum((x - mean) ** 2 for x in pair) / 2)
    assert abs(s.pair_score_std - std) < 1e-6
    assert abs(s.mean_score_a - sum(valid) / 7) < 1e-6
    assert (s.terminal, s.nagari, s.decision_steps, s.games_per_s) == (6, 2, 17, 4.0)
