"""GPU: the sequence training forward (SeqNet.forward_games, python/cugo_seq50.py:
240-265) and the event encoding (encode_events, :91-109) on the native kernels.

encode_events is exact (0/1 planes and small counts).  games_attention writes bf16:
within 2^-8 |ref| + 1e-5 of the fp32 attention of the same bf16 inputs.  The whole
forward is held to the decoder's bar: its error against the reference's fp32
forward no larger (x1.5) than that of the reference under bf16 autocast (+1e-4), at
most 2e-2 of the logit scale, and the argmax equal wherever the top-2 margin
exceeds 4x the error.
"""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from tests import seq_reference as sr

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _golden_hist(golden):
    g = {k: torch.from_numpy(v).to(DEV) for k, v in golden("seq_games").items()}
    return g, SimpleNamespace(events=g["events"], count=g["count"], start=g["start"], seat=g["seat"])


def _random_hist(seed, s_n, length, q_n):
    g = torch.Generator().manual_seed(seed)
    k50 = (1 << 50) - 1
    ev = torch.randint(0, 1 << 62, (s_n, 48, 9), generator=g) & k50
    ev &= torch.randint(0, 2, (s_n, 48, 9), generator=g) * k50  # some empty masks
    ev[..., 8] = torch.randint(0, 2, (s_n, 48), generator=g) | (torch.randint(0, 14, (s_n, 48),
                                                                               generator=g) << 8)
    count = torch.randint(0, length + 1, (s_n,), generator=g)
    count[0] = length
    ev[torch.arange(48).view(1, -1) >= count.view(-1, 1)] = 0
    start = torch.randint(0, 1 << 62, (s_n, 8), generator=g) & k50
    start[:, 6] &= (1 << 12) - 1
    start[:, 7] = torch.randint(0, 9, (s_n,), generator=g) | (torch.randint(0, 5, (s_n,), generator=g) << 8) \
        | (torch.randint(0, 2, (s_n,), generator=g) << 16) | (torch.randint(0, 4, (s_n,), generator=g) << 24) \
        | (torch.randint(0, 4, (s_n,), generator=g) << 32)
    seat = torch.randint(0, 2, (s_n,), generator=g)
    feats = torch.rand((s_n, q_n, 720), generator=g).to(torch.bfloat16).float()
    legal = torch.rand((s_n, q_n, 179), generator=g) < 0.1
    seen = torch.minimum(torch.randint(0, length + 1, (s_n, q_n), generator=g).sort(1).values,
                         count.view(-1, 1))
    t = dict(events=ev, count=count, start=start, seat=seat, features=feats, legal=legal, seen=seen)
    t = {k: v.to(DEV) for k, v in t.items()}
    return t, SimpleNamespace(events=t["events"], count=t["count"], start=t["start"], seat=t["seat"])


def test_encode_events_matches_reference_golden(golden):
    from cugo_b200.seq import encode_events
    g, h = _golden_hist(golden)
    for dtype in (torch.float32, torch.bfloat16):
        tokens, valid = encode_events(h, 48, dtype)
        assert tokens.dtype == dtype
        assert torch.equal(tokens.float(), g["tokens"].float())
        assert torch.equal(valid, g["valid"])


def test_encode_events_matches_restatement_on_random_words():
    from cugo_b200.seq import encode_events
    t, h = _random_hist(1, 300, 40, 4)
    tokens, valid = encode_events(h, 33, torch.float32)
    assert torch.equal(tokens, sr.event_tokens(t["events"], t["seat"], 33))
    assert torch.equal(valid, torch.arange(33, device=DEV).view(1, -1) < t["count"].view(-1, 1))


def _decoder(seed):
    from cugo_b200.seq import SeqDecoder
    return SeqDecoder.from_state_dict(SeqDecoder.random_state(seed=seed), device=DEV)


def _check_forward(out, full, auto):
    err = float((out - full).abs().max())
    err_ref = float((auto - full).abs().max())
    scale = float(full.abs().max())
    assert err <= 1.5 * err_ref + 1e-4, (err, err_ref)
    assert err <= 2e-2 * scale, (err, scale)
    flat, ours = full.reshape(-1, full.shape[-1]), out.reshape(-1, out.shape[-1])
    top2 = flat.topk(2, 1).values
    clear = (top2[:, 0] - top2[:, 1]) > 4 * err
    assert torch.equal(ours.argmax(1)[clear], flat.argmax(1)[clear])


def test_forward_games_matches_reference_golden(golden):
    g, h = _golden_hist(golden)
    out = _decoder(13).forward_games(h, g["features"], g["legal"], g["seen"])
    _check_forward(out, g["games_full"], g["games_autocast"])


@pytest.mark.parametrize("s_n,length,q_n", [(200, 40, 18), (33, 48, 1), (64, 1, 30)])
def test_forward_games_matches_restatement(s_n, length, q_n):
    from cugo_b200.seq import SeqDecoder
    t, h = _random_hist(s_n + length, s_n, length, q_n)
    p = {k: v.to(DEV) for k, v in SeqDecoder.random_state(seed=3).items()}
    args = (t["events"], t["count"], t["start"], t["seat"], t["features"], t["legal"], t["seen"],
            length)
    with torch.no_grad():
        full = sr.forward_games(p, *args)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            auto = sr.forward_games(p, *args).float()
    out = _decoder(3).forward_games(h, t["features"], t["legal"], t["seen"], length=length)
    _check_forward(out, full, auto)


def test_games_attention_matches_fp32():
    from cugo_b200 import load_extension
    ext = load_extension()
    g = torch.Generator().manual_seed(7)
    s_n, length, q_n = 37, 23, 9
    t = 1 + length + q_n
    qkv = torch.randn((s_n * t, 768), generator=g).to(DEV, torch.bfloat16)
    seen = torch.randint(-2, length + 3, (s_n, q_n), generator=g).to(DEV)
    out = ext.games_attention(qkv, s_n, length, q_n, seen.reshape(-1).contiguous())
    # Rebuild per-sequence [t] token order: opening, events, queries.
    rows = torch.cat((torch.arange(s_n).view(-1, 1),
                      s_n + torch.arange(s_n * length).view(s_n, length),
                      s_n + s_n * length + torch.arange(s_n * q_n).view(s_n, q_n)), 1).to(DEV)
    x = qkv.float()[rows]  # [s_n, t, 768]
    q, k, v = (z.reshape(s_n, t, 8, 32).transpose(1, 2) for z in x.chunk(3, -1))
    allowed = torch.zeros(s_n, t, t, dtype=torch.bool, device=DEV)
    allowed[:, :, 0] = True
    allowed[:, 1:length + 1, 1:length + 1] = torch.ones(length, length, dtype=torch.bool,
                                                        device=DEV).tril()
    allowed[:, length + 1:, 1:length + 1] = torch.arange(length, device=DEV).view(1, 1, -1) \
        < seen.unsqueeze(-1)
    allowed[:, length + 1:, length + 1:] = torch.eye(q_n, dtype=torch.bool, device=DEV)
    sc = (q @ k.transpose(-1, -2)) * 32 ** -0.5
    ref = (torch.softmax(sc.masked_fill(~allowed.unsqueeze(1), float("-inf")), -1) @ v)
    ref = ref.transpose(1, 2).reshape(s_n, t, 256)
    got = out.float()[rows]
    diff = (got - ref).abs()
    assert bool((diff <= 2.0 ** -8 * ref.abs() + 1e-5).all()), float(diff.max())
