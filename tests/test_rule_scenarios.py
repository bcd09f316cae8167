"""Known-answer rule scenarios (tests/scenarios.py): each hand-built decision point is
stepped by the reference engine (oracle) and by this engine -- the host build of its
headers on CPU, the kernels on the GPU -- with identical rows and outputs required
after every action, and the rule outcome the reference's own test asserts checked on
the result."""
from __future__ import annotations

import numpy as np
import pytest

from tests import host_engine as he
from tests import scenarios as sc


def _w(row: np.ndarray) -> np.ndarray:
    return row.reshape(-1).view(np.uint64)


def _get(row, word, shift, width):
    return (int(_w(row)[word]) >> shift) & ((1 << width) - 1)


def _has(mask: int, *cards: int) -> bool:
    return all(mask >> c & 1 for c in cards)


def _pile(row, p):
    return int(_w(row)[4 + p])


def _round(row):
    r = _get(row, 18, 32, 8)
    return r if r else 1


def _side0(row):
    v = _get(row, 18, 0, 32)
    return v - (1 << 32) if v >= 1 << 31 else v


C = sc.card


def _check_outcome(name: str, before: np.ndarray, steps: list[tuple]) -> None:
    """The reference test's assertions, on the oracle's result rows."""
    after = steps[-1][0][0]
    status = [int(s[4][0]) for s in steps]
    if name == "neutral_ppuk_capture":
        assert status == [0]
        assert _has(_pile(after, 0), C(3, 0), C(3, 1), C(3, 2), C(3, 3))
        assert bin(_pile(after, 1)).count("1") == 1          # one pi stolen
        assert _get(after, 11, 0, 16) & (1 << 3) == 0         # the neutral ppuk is gone
    elif name == "last_turn_jjok":
        assert status == [0]
        assert _has(_pile(after, 0), C(0, 0), C(0, 1))
        assert _pile(after, 1) == _pile(before, 1)            # no steal on the last turns
    elif name == "last_turn_ppuk":
        assert status == [0]
        assert _get(after, 8, 0, 16) == 0                     # no ppuk stack
        assert _has(_pile(after, 0), C(1, 0))                 # the matched card captured
    elif name == "ppuk_before_last_turn":
        assert status == [0]
        assert _get(after, 8, 0, 16) & (1 << 1)               # the ppuk stack of month 1
    elif name == "last_turn_bonus":
        assert status == [0]
        assert _pile(after, 1) == _pile(before, 1)            # nothing stolen
        assert _has(_pile(after, 0), 48)
    elif name == "first_turn_ttadak":
        assert status == [0]
        assert _has(_pile(after, 0), C(2, 0), C(2, 1), C(2, 2), C(2, 3))
        assert bin(_pile(after, 1)).count("1") == 1           # one pi stolen
        assert _side0(after) == 7 * _round(before)            # first-turn ttadak pays 7
    elif name == "third_ppuk":
        assert status == [0]
        assert _get(after, 16, 8, 8) == 5                     # ended by three ppuk
        assert after[sc.DONE_BYTE] == 1
    elif name == "bonus_replacement_chongtong":
        assert status == [0, 0]
        prompt = steps[0][0][0]
        assert _get(prompt, 15, 32, 8) == 0 and _get(prompt, 15, 48, 16) & 1  # offered
        assert _get(after, 16, 8, 8) == 4                     # bonus-replacement Chongtong
    elif name == "forced_bomb":
        assert status == [3, 0]                               # the single play is not legal
        assert _get(after, 13, 32, 8) == 1                    # one bomb
        assert _has(_pile(after, 0), C(4, 0), C(4, 1), C(4, 2), C(4, 3))
    elif name == "four_card_shake":
        assert status == [0]
        assert _get(after, 14, 0, 16) & (1 << 4)              # shaken with all four
    elif name == "bomb_credit":
        assert status == [0]
        assert _get(after, 13, 48, 8) == 0                    # the credit spent
    else:
        raise AssertionError(name)


@pytest.fixture(scope="module")
def case_rows(oracle):
    base = sc.fresh_row(oracle)
    return {c.name: sc.build(c, base, he) for c in sc.CASES}


def _same(ref, mine, name, k):
    for j, what in enumerate(("rows", "reward", "done", "nagari", "status", "committed")):
        assert np.array_equal(np.asarray(ref[j]), np.asarray(mine[j])), (name, k, what)


@pytest.mark.parametrize("case", sc.CASES, ids=lambda c: c.name)
def test_scenario_on_host_engine(oracle, case_rows, case):
    row = case_rows[case.name][None, :]
    fo, lo, po, do, so = oracle.observe(row)
    fh, lh, ph, dh, sh = he.observe(row)
    assert np.abs(fo - fh).max() <= 1e-6 and np.array_equal(lo, lh)
    assert np.array_equal(so, sh) and np.array_equal(po, ph)
    if case.name == "forced_bomb":
        assert not lo[0, C(4, 0):C(4, 3)].any() and lo[0, 98 + 4]
    if case.name == "four_card_shake":
        assert lo[0, 50 + C(4, 0):50 + C(4, 3) + 1].all()
    ref = sc.play(row, case.actions, oracle.step)
    mine = sc.play(row, case.actions, lambda r, a: he.step(r, a))
    for k, (a, b) in enumerate(zip(ref, mine)):
        _same(a, b, case.name, k)
    _check_outcome(case.name, row[0], ref)


@pytest.mark.gpu
def test_scenarios_on_gpu(ext, oracle, case_rows):
    import torch
    dev = torch.device("cuda:0")
    for case in sc.CASES:
        row = case_rows[case.name][None, :]
        ref = sc.play(row, case.actions, oracle.step)
        states = torch.from_numpy(row.copy()).to(dev)
        for k, a in enumerate(case.actions):
            out = ext.step(states, torch.full((1,), a, dtype=torch.int64, device=dev))
            mine = (states.cpu().numpy(),) + tuple(t.cpu().numpy() for t in out)
            _same(ref[k], mine, case.name, k)
