"""CPU: GAE(lambda) of the PPO iteration (python/cugo_ppo50.py:484-509) against a
per-sequence recursion written out directly."""
from __future__ import annotations

import torch

from cugo_b200.train import gae_advantages


def _direct(values, returns, env_ids, seat, lam):
    out = torch.zeros_like(values)
    seqs: dict[tuple[int, int], list[int]] = {}
    for i in range(values.numel()):
        seqs.setdefault((int(env_ids[i]), int(seat[i])), []).append(i)
    for rows in seqs.values():
        acc = 0.0
        for j in reversed(range(len(rows))):
            r = rows[j]
            nxt = float(values[rows[j + 1]]) if j + 1 < len(rows) else float(returns[r])
            acc = (nxt - float(values[r])) + lam * acc
            out[r] = acc
    return out


def test_gae_matches_the_recursion():
    g = torch.Generator().manual_seed(3)
    # step-major rows: round k holds the games still running
    env_ids, seat = [], []
    alive = list(range(40))
    lengths = torch.randint(1, 30, (40,), generator=g)
    for k in range(30):
        for e in alive:
            if k < int(lengths[e]):
                env_ids.append(e)
                seat.append((e + k) % 2)
    env_ids = torch.tensor(env_ids)
    seat = torch.tensor(seat)
    n = env_ids.numel()
    values = torch.randn(n, generator=g)
    returns = torch.randn(n, generator=g)
    for lam in (0.0, 0.95, 0.5):
        got = gae_advantages(values, returns, env_ids, seat, lam)
        assert torch.allclose(got, _direct(values, returns, env_ids, seat, lam), atol=1e-5)
    assert torch.equal(gae_advantages(values, returns, env_ids, seat, 1.0), returns - values)
