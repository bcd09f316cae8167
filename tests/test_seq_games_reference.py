"""CPU: the test-side restatement of the sequence training forward and of the event
encoding (tests/seq_reference.py) against the reference's own outputs in
tests/golden/seq_games.npz (made by tests/golden/make_seq_games_golden.py)."""
from __future__ import annotations

import numpy as np
import torch

from cugo_b200.seq import SeqDecoder
from tests import seq_reference as sr


def _t(g):
    return {k: torch.from_numpy(v) for k, v in g.items()}


def test_event_tokens_restatement_matches_reference(golden):
    t = _t(golden("seq_games"))
    tokens = sr.event_tokens(t["events"], t["seat"], 48)
    assert torch.equal(tokens, t["tokens"].float())
    assert torch.equal(torch.arange(48).view(1, -1) < t["count"].view(-1, 1), t["valid"])


def test_forward_games_restatement_matches_reference(golden):
    t = _t(golden("seq_games"))
    p = SeqDecoder.random_state(seed=13)
    out = sr.forward_games(p, t["events"], t["count"], t["start"], t["seat"], t["features"],
                           t["legal"], t["seen"], int(t["count"].max()))
    full = t["games_full"]
    assert out.shape == full.shape
    assert float((out - full).abs().max()) <= 1e-4 * float(full.abs().max())
    assert np.isfinite(out.numpy()).all()
