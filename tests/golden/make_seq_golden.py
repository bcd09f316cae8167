"""Golden outputs of the reference's sequence policy (python/cugo_seq50.py SeqNet and
python/cugo_seq_attention50.py decode_attention), imported from the reference tree.

    make -C oracle && python tests/golden/make_seq_golden.py     # needs the reference tree

seq_decode.npz holds, for 32 real game positions played with the oracle engine
(the first 32 games i that do not end at the deal: seed 12345 + i, first player
i & 1; random legal actions from numpy default_rng(5), stopped after
3 + 7j mod 30 decisions for the j-th game or before the step that would finish it):
  games [32], start [32, 8], events [32, 48, 9], count [32], seat [32] (the mover),
  features [32, 720] (bf16-rounded), legal [32, 179]
and the reference's outputs with weights SeqDecoder.random_state(seed=11):
  logits_full      SeqNet.forward in fp32 (CPU)
  logits_autocast  SeqNet.forward under bf16 autocast (CPU)
  logits_inc       start_token/event_token/query_token + cached_step + readout,
                   the wave collector's incremental path, in fp32 (decode
                   attention through its matrix-product path)
  start_tok, event_tok0   start_token and the first event_token, fp32
  att_out          decode_attention(use_triton=False) in fp32 on
                   tests/seq_reference.attention_case(seed=3, n=48, n_rows=64)
  logits_events_full, logits_events_autocast
                   SeqNet("events").forward in fp32 and under bf16 autocast (CPU) with
                   the weights SeqDecoder.random_state(seed=11, mode="events")
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
sys.path.insert(0, str(ROOT / "tests"))

from oracle import ref  # noqa: E402
from seq_reference import attention_case  # noqa: E402

B, MAX_EVENTS, WEIGHT_SEED = 32, 48, 11


def play_positions():
    # The first B games that do not end at the deal (a Chongtong deal finishes at once).
    cand = np.arange(4 * B, dtype=np.int64)
    fresh = ref.create(12345 + cand, cand & 1)
    idx = cand[~ref.observe(fresh)[3]][:B]
    rows = fresh[idx]
    start = ref.start(rows)
    events = np.zeros((B, MAX_EVENTS, 9), dtype=np.int64)
    count = np.zeros(B, dtype=np.int64)
    rng = np.random.default_rng(5)
    target = 3 + (7 * np.arange(B)) % 30
    for i in range(B):
        row = rows[i:i + 1]
        for _ in range(int(target[i])):
            _, legal, _, done, _ = ref.observe(row)
            acts = np.flatnonzero(legal[0])
            if done[0] or acts.size == 0:
                break
            a = np.array([rng.choice(acts)], dtype=np.int64)
            nxt, _, ndone, _, status, committed, ev = ref.step(row, a, events=True)
            assert status[0] == 0
            if ndone[0]:
                break  # keep the position before the finishing step
            if committed[0]:
                events[i, count[i]] = ev[0]
                count[i] += 1
            row = nxt
        rows[i] = row[0]
    features, legal, player, done, _ = ref.observe(rows)
    assert not done.any()
    return idx, start, events, count, player.astype(np.int64), features, legal


def main() -> None:
    sys.path.insert(0, str(REF))
    from cugo_seq50 import HistBatch, KVCache, SeqNet  # the reference's modules
    from cugo_seq_attention50 import decode_attention
    from cugo_b200.seq import SeqDecoder

    games, start, events, count, seat, features, legal = play_positions()
    model = SeqNet("hybrid", 179).eval()
    model.load_state_dict(SeqDecoder.random_state(seed=WEIGHT_SEED), strict=True)
    t = {k: torch.from_numpy(v) for k, v in dict(start=start, events=events, count=count, seat=seat,
                                                   legal=legal).items()}
    feats = torch.from_numpy(features).to(torch.bfloat16).float()
    hist = HistBatch(t["events"], t["count"], t["start"], t["seat"])
    with torch.no_grad():
        logits_full = model(feats, t["legal"], hist)
        with torch.autocast("cpu", dtype=torch.bfloat16):
            logits_autocast = model(feats, t["legal"], hist).float()
        cache = KVCache(model, B, torch.device("cpu"))
        cache.use_triton = False
        start_tok = model.start_token(t["start"], t["seat"])
        model.cached_step(cache, start_tok.clone(), 1)
        cache.length.fill_(1)
        event_tok0 = None
        for e in range(int(count.max())):
            x = model.event_token(t["events"][:, e], t["seat"], torch.full((B,), e, dtype=torch.int64))
            if e == 0:
                event_tok0 = x.clone()
            model.cached_step(cache, x)
            cache.length += (e < t["count"]).long()
        q = model.query_token(feats, t["legal"])
        h = model.cached_step(cache, q, rows=torch.arange(B))
        logits_inc = model.readout(h)
        aq, ak, av, apos, arows = attention_case(seed=3, n=48, n_rows=64)
        att_out = decode_attention(aq, ak, av, apos, use_triton=False, rows=arows)
        events_model = SeqNet("events", 179).eval()
        events_model.load_state_dict(SeqDecoder.random_state(seed=WEIGHT_SEED, mode="events"),
                                     strict=True)
        logits_events_full = events_model(feats, t["legal"], hist)
        with torch.autocast("cpu", dtype=torch.bfloat16):
            logits_events_autocast = events_model(feats, t["legal"], hist).float()
    out = HERE / "seq_decode.npz"
    np.savez_compressed(out, games=games, start=start, events=events, count=count, seat=seat,
                        features=feats.numpy(), legal=legal, logits_full=logits_full.numpy(),
                        logits_autocast=logits_autocast.numpy(), logits_inc=logits_inc.numpy(),
                        start_tok=start_tok.numpy(), event_tok0=event_tok0.numpy(),
                        att_out=att_out.numpy(), logits_events_full=logits_events_full.numpy(),
                        logits_events_autocast=logits_events_autocast.numpy())
    d = (logits_inc - logits_full).abs().max().item()
    print(out.name, out.stat().st_size, "events max", int(count.max()), "inc-vs-full", d)


if __name__ == "__main__":
    main()
