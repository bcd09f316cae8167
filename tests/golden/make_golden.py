"""Generates the committed golden fixtures from the oracle (the reference engine
compiled from its own sources, oracle/_ref/libcugo_ref.so).

    make -C oracle && python tests/golden/make_golden.py

Fixtures (numpy .npz, compressed):
  config0.npz   seeded random-legal games 0..4095 (seed 12345 + i, first i & 1):
                per-game FNV-1a event hash, reward0, decisions, events, status,
                final_points, and the first 256 final rows
  create.npz    512 fresh rows from three seed families (config, make_seeds, random)
  steps.npz     512 mid-game rows with their observe outputs, a random action each
                (some illegal), the step outputs, events and stepped rows
  roots.npz     config-2 roots 0..255 and their first 4 branch actions
The GPU tests compare the CUDA path against these without needing the oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import ref  # noqa: E402

OUT = Path(__file__).resolve().parent
SIGNED_GOLDEN = -7046029254386353131
SEED_BASE = 0x243F6A8885A308D3


def seed_families(n: int) -> tuple[np.ndarray, np.ndarray]:
    idx = np.arange(n, dtype=np.int64)
    with np.errstate(over="ignore"):
        a = 12345 + idx
        b = idx * np.int64(SIGNED_GOLDEN) + np.int64(SEED_BASE)
    c = np.random.default_rng(2024).integers(-2**63, 2**63 - 1, size=n, dtype=np.int64)
    seeds = np.concatenate([a, b, c])
    first = np.concatenate([idx & 1, idx & 1, (idx + 1) & 1])
    return seeds, first


def mid_game_rows(n: int, rng: np.random.Generator) -> np.ndarray:
    """Rows after a random number of random-legal decisions (incl. pending choices)."""
    seeds, first = seed_families(n)
    rows = ref.create(seeds, first)
    target = rng.integers(0, 24, size=rows.shape[0])
    for d in range(40):
        _, legal, _, done, _ = ref.observe(rows)
        live = (~done) & (target > d)
        if not live.any():
            break
        cnt = legal.sum(1)
        pick = np.minimum((rng.random(rows.shape[0]) * np.maximum(cnt, 1)).astype(np.int64),
                          np.maximum(cnt - 1, 0))
        actions = np.argmax(np.cumsum(legal, 1) > pick[:, None], 1).astype(np.int64)
        nxt = ref.step(rows, actions)[0]
        rows = np.where(live[:, None], nxt, rows)
    return rows


def main() -> None:
    rng = np.random.default_rng(7)
    r = ref.rollout_random(0, 4096, seed_base=12345, max_decisions=256)
    final_points = np.array([ref.settle(row)[3] for row in r["final_rows"]], dtype=np.int64)
    np.savez_compressed(OUT / "config0.npz", hashes=r["hashes"], reward0=r["reward0"],
                        decisions=r["decisions"], events=r["events"],
                        last_status=r["last_status"], final_points=final_points,
                        final_rows_head=r["final_rows"][:256])

    seeds, first = seed_families(512 // 3 + 1)
    seeds, first = seeds[:512], first[:512]
    np.savez_compressed(OUT / "create.npz", seeds=seeds, first=first, rows=ref.create(seeds, first))

    rows = mid_game_rows(171, rng)[:512]
    features, legal, player, done, status = ref.observe(rows)
    cnt = legal.sum(1)
    pick = np.minimum((rng.random(rows.shape[0]) * np.maximum(cnt, 1)).astype(np.int64),
                      np.maximum(cnt - 1, 0))
    actions = np.argmax(np.cumsum(legal, 1) > pick[:, None], 1).astype(np.int64)
    bad = rng.random(rows.shape[0]) < 0.1
    actions[bad] = rng.integers(-2, 181, size=int(bad.sum()))
    nxt, reward, sdone, nagari, sstatus, committed, events = ref.step(rows, actions, events=True)
    np.savez_compressed(OUT / "steps.npz", rows=rows, features=features, legal=legal,
                        player=player, done=done, status=status, actions=actions, next_rows=nxt,
                        reward=reward, step_done=sdone, nagari=nagari, step_status=sstatus,
                        committed=committed, events=events, start=ref.start(rows),
                        stock=ref.stock(rows), hands=ref.hands(rows))

    roots = ref.branch_roots(256)
    ids, acts = ref.branch_actions(roots, 4)
    np.savez_compressed(OUT / "roots.npz", roots=roots, ids=ids, actions=acts)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
