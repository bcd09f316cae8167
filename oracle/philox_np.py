"""Vectorised numpy Philox4x32-10 (Salmon et al., SC'11) and the samplers' Gumbel noise
(TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: the expectations of tests/ and the noise
of bench.py's CPU baseline; the product draws its noise on the device)."""
from __future__ import annotations

import numpy as np

M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    c = [np.asarray(x, dtype=np.uint64) & MASK for x in (c0, c1, c2, c3)]
    k0 = np.asarray(k0, dtype=np.uint64) & MASK
    k1 = np.asarray(k1, dtype=np.uint64) & MASK
    for _ in range(10):
        p0 = np.uint64(M0) * c[0]
        p1 = np.uint64(M1) * c[2]
        c = [(p1 >> np.uint64(32)) ^ c[1] ^ k0, p1 & MASK, (p0 >> np.uint64(32)) ^ c[3] ^ k1, p0 & MASK]
        k0 = (k0 + np.uint64(W0)) & MASK
        k1 = (k1 + np.uint64(W1)) & MASK
    return [x.astype(np.uint32) for x in c]


def gumbel_noise(game: np.ndarray, decision: np.ndarray, seed_base: int) -> np.ndarray:
    """[n, 179] Gumbel noise of the sampler kernel's addressing."""
    game = game.astype(np.uint64)
    seed = (game + np.uint64(seed_base)) & np.uint64(0xFFFFFFFFFFFFFFFF)
    out = np.zeros((game.shape[0], 180), dtype=np.float64)
    for blk in range(45):
        words = philox4x32_10(game & MASK, game >> np.uint64(32), decision.astype(np.uint64),
                              np.uint64(3 | (blk << 8)), seed & MASK, seed >> np.uint64(32))
        for j in range(4):
            u = ((words[j] >> np.uint32(8)).astype(np.float64) + 0.5) / 16777216.0
            out[:, 4 * blk + j] = -np.log(-np.log(u))
    return out[:, :179]
