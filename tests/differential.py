"""Step-by-step differential play against the oracle.

`play_against_oracle(impl, ...)` drives seeded games with uniformly random legal
actions (plus injected illegal actions) through an implementation under test and
through the oracle, comparing at every decision: observation features (1e-6, the
reference's own tolerance for the log2f feature, tests/cuda_torch50_test.cu:135),
legal masks, players, done flags, statuses, then the stepped rows byte for byte
and every step output and event record exactly.

`impl` exposes numpy-in/numpy-out create/observe/step(events=True)/start/stock
like oracle.ref does.
"""
from __future__ import annotations

import numpy as np

SIGNED_GOLDEN = -7046029254386353131
SEED_BASE = 0x243F6A8885A308D3

# Named byte ranges of a row, for readable mismatch reports.
FIELDS = [("hand0", 0, 8), ("hand1", 8, 8), ("floor", 16, 8), ("stock", 24, 8), ("pile0", 32, 8),
          ("pile1", 40, 8), ("rng", 48, 8), ("flip_bonus", 56, 8), ("ppuk", 64, 2),
          ("owner1", 66, 2), ("ppuk_b2", 68, 2), ("ppuk_b3", 70, 2), ("turn", 72, 2),
          ("actor", 74, 1), ("phase", 75, 1), ("played", 76, 1), ("drawn", 77, 1),
          ("mission", 80, 8), ("neutral", 88, 2), ("go", 96, 2), ("last_go", 98, 2),
          ("gostop_actor", 100, 1), ("winner", 101, 1), ("gukjin", 102, 1), ("shaken", 104, 4),
          ("bombs", 108, 2), ("credits", 110, 2), ("shaken4", 112, 4), ("ppuk_count", 120, 2),
          ("ppuk_streak", 122, 2), ("chong_actor", 124, 1), ("chong_months", 126, 2),
          ("end", 128, 2), ("end_points", 136, 8), ("side0", 144, 4), ("round", 148, 1),
          ("mission_meta", 149, 4), ("held", 160, 16), ("shown", 176, 16), ("pending", 192, 32),
          ("counters", 224, 14), ("status", 238, 1), ("done", 239, 1), ("nagari", 240, 1)]


def field_diff(a: np.ndarray, b: np.ndarray) -> list:
    return [(n, a[o:o + k].tobytes().hex(), b[o:o + k].tobytes().hex())
            for n, o, k in FIELDS if a[o:o + k].tobytes() != b[o:o + k].tobytes()]


def seeds_for(family: int, n: int, salt: int = 0) -> tuple[np.ndarray, np.ndarray]:
    idx = np.arange(n, dtype=np.int64)
    with np.errstate(over="ignore"):
        if family == 0:
            seeds = 12345 + idx + salt
        elif family == 1:
            seeds = (idx + salt) * np.int64(SIGNED_GOLDEN) + np.int64(SEED_BASE)
        else:
            seeds = np.random.default_rng(salt).integers(-2**63, 2**63 - 1, size=n, dtype=np.int64)
    return seeds, (idx + salt) & 1


def random_legal(legal: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    cnt = legal.sum(1)
    pick = np.minimum((rng.random(legal.shape[0]) * np.maximum(cnt, 1)).astype(np.int64),
                      np.maximum(cnt - 1, 0))
    return np.argmax(np.cumsum(legal, 1) > pick[:, None], 1).astype(np.int64)


def play_against_oracle(impl, oracle, n: int, family: int, salt: int, max_decisions: int = 64,
                        inject: float = 0.03) -> dict:
    seeds, first = seeds_for(family, n, salt)
    rows_o = oracle.create(seeds, first)
    rows_i = impl.create(seeds, first)
    assert np.array_equal(rows_o, rows_i), ("create", field_diff(rows_o[0], rows_i[0]))
    rng = np.random.default_rng(salt + 17)
    kinds = np.zeros(8, dtype=np.int64)
    steps = 0
    for d in range(max_decisions):
        fo = oracle.observe(rows_o)
        fi = impl.observe(rows_i)
        err = np.abs(fo[0] - fi[0]).max(1)
        bad = np.nonzero(err > 1e-6)[0]
        assert bad.size == 0, ("features", d, bad[:5],
                               np.nonzero(np.abs(fo[0][bad[0]] - fi[0][bad[0]]) > 1e-6)[0][:10])
        for k, name in enumerate(["legal", "player", "done", "status"], start=1):
            m = fo[k] != fi[k]
            if m.ndim > 1:
                m = m.any(1)
            assert not m.any(), (name, d, np.nonzero(m)[0][:5])
        assert np.array_equal(oracle.start(rows_o), impl.start(rows_i)), ("start", d)
        assert np.array_equal(oracle.stock(rows_o), impl.stock(rows_i)), ("stock", d)
        # Decision kinds seen (one-hot at 447..451, Gukjin flag at 552).
        kinds[1:6] += (fo[0][:, 447:452] == 1.0).sum(0)
        kinds[7] += int((fo[0][:, 552] == 1.0).sum())
        live = ~fo[3]
        if not live.any():
            break
        steps += int(live.sum())
        actions = random_legal(fo[1], rng)
        inj = rng.random(n) < inject
        actions[inj] = rng.integers(-3, 182, size=int(inj.sum()))
        so = oracle.step(rows_o, actions, events=True)
        si = impl.step(rows_i, actions, events=True)
        for k, name in enumerate(["rows", "reward", "done", "nagari", "status", "committed",
                                  "events"]):
            m = so[k] != si[k]
            if m.ndim > 1:
                m = m.any(1)
            if m.any():
                i = int(np.nonzero(m)[0][0])
                detail = field_diff(so[0][i], si[0][i]) if k == 0 else (so[k][i], si[k][i])
                raise AssertionError((name, "decision", d, "row", i, "action", int(actions[i]),
                                      detail))
        rows_o, rows_i = so[0], si[0]
    return dict(steps=steps, kinds=kinds, done=float(rows_o[:, 239].mean()))
