"""Golden outputs of the reference's sequence training forward and event encoding
(python/cugo_seq50.py SeqNet.forward_games :240-265, encode_events :91-109),
imported from the reference tree.

    make -C oracle && python tests/golden/make_seq_games_golden.py   # needs the reference tree

seq_games.npz holds 6 complete games played with the oracle engine (game i: seed
20000 + i, first player i & 1; random legal actions from numpy default_rng(9)),
read as 12 (game, seat) sequences, sequence 2i + seat:
  start [12, 8], events [12, 48, 9], count [12] (the game's events), seat [12],
  features [12, Q, 720] (bf16-rounded), legal [12, Q, 179], seen [12, Q] (events
  visible at each of the seat's decisions; padded decisions have seen 0, zero
  features and no legal action)
and, with weights SeqDecoder.random_state(seed=13):
  games_full      SeqNet.forward_games in fp32 (CPU)
  games_autocast  the same under bf16 autocast (CPU)
  tokens, valid   encode_events(hist, 48, float32) of the 12 sequences
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle.build import reference_root  # noqa: E402

REF = reference_root() / "python"

from oracle import ref  # noqa: E402

GAMES, MAX_EVENTS, WEIGHT_SEED = 6, 48, 13


def play_games():
    seeds = 20000 + np.arange(GAMES, dtype=np.int64)
    rows = ref.create(seeds, np.arange(GAMES, dtype=np.int64) & 1)
    start = ref.start(rows)
    events = np.zeros((GAMES, MAX_EVENTS, 9), dtype=np.int64)
    count = np.zeros(GAMES, dtype=np.int64)
    decisions = [[[], []] for _ in range(GAMES)]  # per game, per seat: (features, legal, seen)
    rng = np.random.default_rng(9)
    for i in range(GAMES):
        row = rows[i:i + 1]
        for _ in range(200):
            features, legal, player, done, _ = ref.observe(row)
            if done[0]:
                break
            decisions[i][int(player[0])].append((features[0], legal[0], int(count[i])))
            a = np.array([rng.choice(np.flatnonzero(legal[0]))], dtype=np.int64)
            row, _, _, _, status, committed, ev = ref.step(row, a, events=True)
            assert status[0] == 0
            if committed[0]:
                events[i, count[i]] = ev[0]
                count[i] += 1
        assert ref.observe(row)[3][0]
    q = max(len(d) for g in decisions for d in g)
    s = 2 * GAMES
    feats = np.zeros((s, q, 720), dtype=np.float32)
    legal = np.zeros((s, q, 179), dtype=bool)
    seen = np.zeros((s, q), dtype=np.int64)
    for i in range(GAMES):
        for seat in (0, 1):
            for j, (f, l, n) in enumerate(decisions[i][seat]):
                feats[2 * i + seat, j], legal[2 * i + seat, j], seen[2 * i + seat, j] = f, l, n
    return (np.repeat(start, 2, axis=0), np.repeat(events, 2, axis=0), np.repeat(count, 2),
            np.tile(np.array([0, 1], dtype=np.int64), GAMES), feats, legal, seen)


def main() -> None:
    sys.path.insert(0, str(REF))
    from cugo_seq50 import HistBatch, SeqNet, encode_events  # the reference's modules
    from cugo_b200.seq import SeqDecoder

    start, events, count, seat, feats, legal, seen = play_games()
    model = SeqNet("hybrid", 179).eval()
    model.load_state_dict(SeqDecoder.random_state(seed=WEIGHT_SEED), strict=True)
    f = torch.from_numpy(feats).to(torch.bfloat16).float()
    hist = HistBatch(torch.from_numpy(events), torch.from_numpy(count), torch.from_numpy(start),
                     torch.from_numpy(seat))
    with torch.no_grad():
        full = model.forward_games(hist, f, torch.from_numpy(legal), torch.from_numpy(seen))
        with torch.autocast("cpu", dtype=torch.bfloat16):
            auto = model.forward_games(hist, f, torch.from_numpy(legal), torch.from_numpy(seen)).float()
        tokens, valid = encode_events(hist, MAX_EVENTS, torch.float32)
    out = HERE / "seq_games.npz"
    np.savez_compressed(out, start=start, events=events, count=count, seat=seat,
                        features=f.numpy(), legal=legal, seen=seen, games_full=full.numpy(),
                        games_autocast=auto.numpy(), tokens=tokens.numpy().astype(np.uint8),
                        valid=valid.numpy())
    print(out.name, out.stat().st_size, "events", count.tolist(), "queries", seen.shape[1],
          "auto-vs-full", float((auto - full).abs().max()))


if __name__ == "__main__":
    main()
