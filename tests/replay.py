"""Replays recorded self-play actions on the oracle engine (TEST INFRASTRUCTURE ONLY).

play_batch(..., actions_log=log) records the action every game chose at each of its
decisions.  Dealing the same games in the reference's engine (oracle/_ref) and
stepping them with those actions must reproduce the final rewards, the nagari flags
and the decision counts bit for bit."""
from __future__ import annotations

import numpy as np


def replay_on_oracle(oracle, game_index: np.ndarray, log: np.ndarray, seed_base: int = 12345):
    """Returns (reward0 f32 [g], nagari bool [g], decisions int [g], bad_status int)."""
    g = game_index.shape[0]
    rows = oracle.create(game_index + seed_base, game_index & 1)
    reward0 = np.zeros(g, dtype=np.float32)
    nagari = np.zeros(g, dtype=bool)
    decisions = np.zeros(g, dtype=np.int64)
    live = ~oracle.observe(rows)[3]
    bad = 0
    for d in range(log.shape[1]):
        if not live.any():
            break
        sel = np.nonzero(live)[0]
        new_rows, r, done, nag, status, _ = oracle.step(rows[sel], log[sel, d])
        bad += int((status != 0).sum())
        rows[sel] = new_rows
        decisions[sel] += 1
        fin = sel[done]
        reward0[fin] = r[done]
        nagari[fin] = nag[done]
        live[fin] = False
    return reward0, nagari, decisions, bad
