"""numpy restatement of the redeal (TEST INFRASTRUCTURE ONLY).

The reference's _redeal (python/cugo_ppo50.py:125-149) on int64 words of TorchEnv50
rows (offsets python/cugo_ppo50.py:109): the observer's opponent keeps the hand
cards a shake revealed and gets the rest — as many as before — uniformly from the
cards the observer cannot see (those hand cards and the stock); the stock is what
remains; `held` follows the new hand; the stock draw seed is replaced.  The random
source is the device kernel's: Philox4x32-10 counter {row lo, row hi, attempt,
8 + k / 4}, word k % 4, picks the floor(word * left / 2^32)-th remaining card;
the seed word is ((w0 << 32 | w1) >> 1) - 2^62 from counter {row lo, row hi,
attempt, 7}.
"""
from __future__ import annotations

import numpy as np

from oracle.philox_np import philox4x32_10

HAND0, HAND1, STOCK, RNG, HELD0, HELD1, REV0, REV1 = 0, 1, 3, 6, 20, 21, 22, 23


def _bits(mask: int) -> list[int]:
    return [c for c in range(64) if (mask >> c) & 1]


def redeal(rows: np.ndarray, seats: np.ndarray, seed: int, attempt: int,
           counters: np.ndarray | None = None) -> np.ndarray:
    """Redealt copies of [n, 248] uint8 rows for observer seats [n]; row i draws
    with Philox counter counters[i] (default i)."""
    out = np.ascontiguousarray(rows, dtype=np.uint8).copy()
    words = out.view(np.uint64)
    n = out.shape[0]
    idx = (np.arange(n) if counters is None else np.asarray(counters)).astype(np.uint64)
    key = np.uint64(seed & (2**64 - 1))
    k0, k1 = key & np.uint64(0xFFFFFFFF), key >> np.uint64(32)
    lo, hi = idx & np.uint64(0xFFFFFFFF), idx >> np.uint64(32)
    draws = [philox4x32_10(lo, hi, attempt, 8 + b, k0, k1) for b in range(13)]  # <= 52 picks
    sw = philox4x32_10(lo, hi, attempt, 7, k0, k1)
    for i in range(n):
        s0 = int(seats[i]) == 0
        hw, held_w, rev_w = (HAND1, HELD1, REV1) if s0 else (HAND0, HELD0, REV0)
        hand, stock = int(words[i, hw]), int(words[i, STOCK])
        fixed = hand & int(words[i, rev_w])
        held = int(words[i, held_w])
        free = hand & ~fixed
        left = free | stock
        picked = 0
        remaining = bin(left).count("1")
        for k in range(bin(free).count("1")):
            word = int(draws[k >> 2][k & 3][i])
            card = _bits(left)[(word * remaining) >> 32]
            picked |= 1 << card
            left &= ~(1 << card)
            remaining -= 1
        new_hand = fixed | picked
        words[i, STOCK] = np.uint64((free | stock) & ~picked)
        words[i, hw] = np.uint64(new_hand)
        words[i, held_w] = np.uint64((held & ~hand) | new_hand)
        bits63 = ((int(sw[0][i]) << 32) | int(sw[1][i])) >> 1
        words[i, RNG] = np.uint64((bits63 - (1 << 62)) & (2**64 - 1))
    return out


def redeal_worlds(oracle, states: np.ndarray, env_rows: np.ndarray, seats: np.ndarray, worlds: int,
                  seed: int, tries: int):
    """The reference's redeal_worlds (python/cugo_ppo50.py:152-177) with the redeal
    above: world row w = k * R + b starts as states[env_rows[b]]; attempt a redeals
    it with counter w and is kept when the oracle's features and legal mask of the
    observer equal the real deal's.  Returns (rows, attempt kept or -1)."""
    base = np.ascontiguousarray(states[env_rows])
    out = np.tile(base, (worlds, 1))
    seat_k = np.tile(np.asarray(seats), worlds)
    f0, l0 = oracle.observe(base, threads=1)[:2]
    ref_f, ref_l = np.tile(f0, (worlds, 1)), np.tile(l0, (worlds, 1))
    kept = np.full(out.shape[0], -1, dtype=np.int8)
    todo = np.arange(out.shape[0])
    for a in range(tries):
        if todo.size == 0:
            break
        cand = redeal(out[todo], seat_k[todo], seed, a, counters=todo)
        f, l = oracle.observe(cand, threads=1)[:2]
        good = (f == ref_f[todo]).all(1) & (l == ref_l[todo]).all(1)
        out[todo[good]] = cand[good]
        kept[todo[good]] = a
        todo = todo[~good]
    return out, kept
