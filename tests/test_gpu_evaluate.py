"""GPU: the fused paired evaluator (python/cugo_eval50.py:137-361) against the
reference's loop restated over the same ops and policy modules, and the window GEMM
it runs the policies with."""
from __future__ import annotations

import pytest
import torch

from tests import eval_reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _actor(seed: int, activation: str = "silu"):
    from cugo_b200.ppo import FusedResidualMlp
    torch.manual_seed(seed)
    net = FusedResidualMlp(720, 179, 256, 2, activation).to(DEV)
    with torch.no_grad():  # a non-trivial policy: every layer random
        for p in net.parameters():
            p.copy_(torch.randn_like(p) * (1.0 / p.shape[-1]) ** 0.5)
    return net


def test_window_gemm_writes_only_the_window(ext):
    g = torch.Generator().manual_seed(0)
    m, n, k = 1000, 256, 512
    a = torch.randn((m, k), generator=g).to(DEV, torch.bfloat16)
    w = (torch.randn((n, k), generator=g) / k ** 0.5).to(DEV, torch.bfloat16)
    b = torch.randn(n, generator=g).to(DEV)
    full = ext.linear(a, w, b, act=2)
    for r0, rows in ((0, 1000), (130, 300), (517, 0), (999, 1), (900, 500)):
        out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device=DEV)
        win = torch.tensor([r0, rows], dtype=torch.int32, device=DEV)
        ext.linear(a, w, b, act=2, out=out, window=win)
        end = min(m, r0 + rows)
        assert torch.equal(out[r0:end], full[r0:end])
        assert bool((out[:r0] == 7.0).all())
        tail = min(m, r0 + ((rows + 127) // 128) * 128)
        assert bool((out[tail:] == 7.0).all())


@pytest.mark.parametrize("pairs,seed_offset", [(1500, 910000000), (777, 5)])
def test_paired_eval_matches_the_reference_loop(ext, pairs, seed_offset):
    from cugo_b200.evaluate import evaluate_paired
    a, b = _actor(1), _actor(2)
    ref = eval_reference.evaluate_paired(ext, a, b, pairs, seed_offset, 128)
    for graphs in (True, False):
        s = evaluate_paired(ext, a, b, pairs, seed_offset, 128, graphs=graphs)
        assert (s.pairs, s.games, s.evaluated_pairs, s.evaluated_games, s.predecision_excluded) == (
            ref["pairs"], ref["games"], ref["evaluated_pairs"], ref["evaluated_games"],
            ref["predecision_excluded"])
        assert (s.a_wins, s.b_wins, s.draws) == (ref["a_wins"], ref["b_wins"], ref["draws"])
        assert (s.a_p0_wins, s.a_p0_losses, s.a_p0_draws) == ref["a_p0"]
        assert (s.a_p1_wins, s.a_p1_losses, s.a_p1_draws) == ref["a_p1"]
        assert (s.pair_wins, s.pair_losses, s.pair_draws) == ref["pair"]
        assert (s.terminal, s.nagari, s.decision_steps) == (ref["terminal"], ref["nagari"],
                                                            ref["decision_steps"])
        assert s.mean_score_a == ref["mean_score_a"]
        assert s.mean_pair_score_a == ref["mean_pair_score_a"]
        assert s.pair_score_std == ref["pair_score_std"]
        assert s.pair_score_ci95_low == ref["pair_score_ci95_low"]


def test_self_play_is_balanced_and_sampling_runs(ext):
    from cugo_b200.evaluate import evaluate_paired, match
    a = _actor(3, "relu")
    s = evaluate_paired(ext, a, a, 1000, 11, 128)
    # The same policy on both sides of every deal: each pair's two games mirror.
    assert s.a_wins + s.b_wins + s.draws == s.evaluated_games
    assert s.mean_pair_score_a == 0.0 and s.pair_score_std == 0.0
    s2 = evaluate_paired(ext, a, _actor(4), 600, 3, 128, sample_a=True, sample_b=False)
    assert s2.evaluated_games > 1000 and s2.decision_steps > 10
    r = match(ext, a, _actor(4), 1000, 400, 910000000, sample=False)
    assert r["pairs"] <= 1000 and r["lo"] <= r["score"] <= r["hi"]
