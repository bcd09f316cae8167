"""CPU: the redeal restatement (tests/redeal_reference.py) keeps the reference's
invariants (python/cugo_ppo50.py:125-177) on mid-game rows of the oracle engine:
cards conserved, the observer's hand and the shaken cards kept, `held` following
the new hand, the observer's view unchanged in nearly every world, and the new
hand a uniform draw from the cards the observer cannot see."""
from __future__ import annotations

import numpy as np

from tests import redeal_reference as rr

ROOTS = 512


def _words(rows):
    return np.ascontiguousarray(rows).view(np.uint64).astype(np.int64)


def test_redeal_invariants(oracle):
    roots = oracle.branch_roots(ROOTS, seed_base=777, threads=1)
    _, _, players, done, _ = oracle.observe(roots, threads=1)
    roots, seats = roots[~done], players[~done].astype(np.int64)
    new = rr.redeal(roots, seats, seed=5, attempt=0)
    a, b = _words(roots), _words(new)
    opp = np.where(seats == 0, rr.HAND1, rr.HAND0)
    mine = np.where(seats == 0, rr.HAND0, rr.HAND1)
    held = np.where(seats == 0, rr.HELD1, rr.HELD0)
    rev = np.where(seats == 0, rr.REV1, rr.REV0)
    r = np.arange(a.shape[0])
    # Only the opponent's hand and held words, the stock and the stock seed change.
    changed = np.ones(31, dtype=bool)
    for i in range(a.shape[0]):
        keep = changed.copy()
        keep[[opp[i], held[i], rr.STOCK, rr.RNG]] = False
        assert np.array_equal(a[i, keep], b[i, keep])
    assert np.array_equal(a[r, mine], b[r, mine])
    assert np.array_equal(a[r, opp] | a[:, rr.STOCK], b[r, opp] | b[:, rr.STOCK])
    assert not np.any(b[r, opp] & b[:, rr.STOCK])
    pc = np.vectorize(lambda x: bin(int(x) & (2**64 - 1)).count("1"))
    assert np.array_equal(pc(a[r, opp]), pc(b[r, opp]))
    fixed = a[r, opp] & a[r, rev]
    assert np.array_equal(b[r, opp] & fixed, fixed)
    assert np.array_equal(b[r, held], (a[r, held] & ~a[r, opp]) | b[r, opp])
    assert np.all((b[:, rr.RNG] >= -2**62) & (b[:, rr.RNG] < 2**62))
    assert np.mean(a[r, opp] != b[r, opp]) > 0.9
    # The observer's features and legal actions survive the redeal in nearly every row.
    f0, l0 = oracle.observe(roots, threads=1)[:2]
    f1, l1 = oracle.observe(new, threads=1)[:2]
    same = (f0 == f1).all(1) & (l0 == l1).all(1)
    assert same.mean() > 0.85


def test_redeal_draw_is_uniform(oracle):
    roots = oracle.branch_roots(64, seed_base=99, threads=1)
    _, _, players, done, _ = oracle.observe(roots, threads=1)
    row = roots[~done][:1]
    seat = players[~done][:1].astype(np.int64)
    w = _words(row)[0]
    opp = rr.HAND1 if seat[0] == 0 else rr.HAND0
    rev = rr.REV1 if seat[0] == 0 else rr.REV0
    free = int(w[opp]) & ~(int(w[opp]) & int(w[rev]))
    unknown = [c for c in range(50) if ((free | int(w[rr.STOCK])) >> c) & 1]
    count = bin(free & (2**64 - 1)).count("1")
    trials = 4000
    rows = np.repeat(row, trials, axis=0)  # Philox counter is the row index: independent draws
    hits = np.zeros(50)
    for h in _words(rr.redeal(rows, np.repeat(seat, trials), seed=11, attempt=0))[:, opp]:
        for c in unknown:
            hits[c] += (int(h) >> c) & 1
    p = count / len(unknown)
    expect = trials * p
    sd = (trials * p * (1 - p)) ** 0.5
    assert np.all(np.abs(hits[unknown] - expect) < 5 * sd)
