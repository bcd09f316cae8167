"""The engine's rule code (compiled for the host from the same headers the CUDA
kernels use) against the oracle, row by row, on CPU."""
from __future__ import annotations

import numpy as np
import pytest

from tests import differential as dif
from tests import host_engine as he


@pytest.mark.parametrize("family,salt", [(0, 0), (1, 5), (2, 9)])
def test_random_play_matches_oracle(oracle, family, salt):
    stats = dif.play_against_oracle(he, oracle, n=4096, family=family, salt=salt)
    assert stats["done"] > 0.99
    # Primary, Go/Stop, played-card and drawn-card floor choices and the Gukjin
    # prompt all occur; the bonus-replacement Chongtong prompt (kind 3) is rare
    # and is required on the first family.
    required = (1, 2, 3, 4, 5, 7) if family == 0 else (1, 2, 4, 5, 7)
    assert all(stats["kinds"][k] > 0 for k in required), stats["kinds"]


def test_single_action_legality_matches_the_mask():
    """The step checks one action's legality without building the legal mask; on every
    decision of seeded random games (and on rows with a pile of specials: shakes,
    bombs, grenades, credits) it agrees with the mask for all 256 action values."""
    seeds, first = dif.seeds_for(0, 2048, 0)
    rows = he.create(seeds, first)
    rng = np.random.default_rng(7)
    checked = 0
    for _ in range(40):
        assert (he.legal_check(rows) == -1).all()
        checked += rows.shape[0]
        _, legal, _, done, _ = he.observe(rows)
        live = ~done & legal.any(1)
        if not live.any():
            break
        rows = rows[live]
        legal = legal[live]
        # Prefer special plays (98..122) when offered, so their rules are exercised.
        u = rng.random(legal.shape) + np.where(np.arange(179) >= 98, 0.5, 0.0) * (rng.random() < 0.5)
        actions = np.where(legal, u, -1.0).argmax(1).astype(np.int64)
        rows = he.step(rows, actions)[0]
    assert checked > 40_000


def test_golden_steps(golden):
    g = golden("steps")
    f, legal, player, done, status = he.observe(g["rows"])
    assert np.abs(f - g["features"]).max() <= 1e-6
    assert np.array_equal(legal, g["legal"])
    assert np.array_equal(player, g["player"]) and np.array_equal(done, g["done"])
    assert np.array_equal(status, g["status"])
    rows, reward, sdone, nagari, sstatus, committed, events = he.step(g["rows"], g["actions"],
                                                                      events=True)
    assert np.array_equal(rows, g["next_rows"])
    assert np.array_equal(reward, g["reward"]) and np.array_equal(sdone, g["step_done"])
    assert np.array_equal(nagari, g["nagari"]) and np.array_equal(sstatus, g["step_status"])
    assert np.array_equal(committed, g["committed"]) and np.array_equal(events, g["events"])
    assert np.array_equal(he.start(g["rows"]), g["start"])
    assert np.array_equal(he.stock(g["rows"]), g["stock"])


def test_golden_create(golden):
    c = golden("create")
    assert np.array_equal(he.create(c["seeds"], c["first"]), c["rows"])


def _edit(rows: np.ndarray, offset: int, dtype, value) -> np.ndarray:
    rows = rows.copy()
    view = rows[:, offset:offset + np.dtype(dtype).itemsize].view(dtype)
    view[:] = value
    return rows


def test_exhausted_stock_edge_cases(oracle):
    """Rows whose stock holds only bonus cards or nothing: a card play cannot
    flip, the step fails with the stock-empty status and leaves the pending
    record active, and observe reports the failed probe (postchance50.h:279-283,
    torch50.h:247-261)."""
    seeds, first = dif.seeds_for(2, 256, 3)
    rows = oracle.create(seeds, first)
    live = rows[:, 239] == 0
    rows = rows[live]
    bonus_only = _edit(rows, 24, np.uint64, np.uint64(3 << 48))
    for case in (bonus_only, _edit(rows, 24, np.uint64, np.uint64(0))):
        case = oracle.canonicalize(case)
        fo, fi = oracle.observe(case), he.observe(case)
        assert np.abs(fo[0] - fi[0]).max() <= 1e-6
        for k in range(1, 5):
            assert np.array_equal(fo[k], fi[k])
        actions = np.nonzero(fo[1][0])[0]
        acts = np.full(case.shape[0], actions[0] if actions.size else 0, dtype=np.int64)
        acts[::3] = np.arange(0, case.shape[0], 3) % 179
        so = oracle.step(case, acts, events=True)
        si = he.step(case, acts, events=True)
        for a, b in zip(so, si):
            assert np.array_equal(a, b)
        # After a failed flip, observe/step report the probe status again.
        so2, si2 = oracle.observe(so[0]), he.observe(si[0])
        for a, b in zip(so2, si2):
            assert np.allclose(a, b, atol=1e-6) if a.dtype == np.float32 else np.array_equal(a, b)


def test_finished_rows_report_game_finished(oracle):
    r = oracle.rollout_random(0, 256)
    rows = r["final_rows"]
    so = oracle.step(rows, np.zeros(256, dtype=np.int64))
    si = he.step(rows, np.zeros(256, dtype=np.int64))
    for a, b in zip(so, si):
        assert np.array_equal(a, b)
    assert (si[4] == 9).all()
    # A game decided at the deal (Chongtong) took no step, so its rollout reward
    # is 0; every other game reports its settled reward again.
    played = r["decisions"] > 0
    assert np.array_equal(si[1].astype(np.int64)[played], r["reward0"][played])
