"""GPU: the Gumbel-max sampler against a numpy restatement of its definition."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.philox_np import gumbel_noise

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _inputs(m=4096, seed=0):
    rng = np.random.default_rng(seed)
    logits = rng.normal(0, 3, size=(m, 180)).astype(np.float32)
    legal = rng.random((m, 179)) < 0.2
    legal[np.arange(m), rng.integers(0, 179, size=m)] = True
    legal[5] = False  # a row without legal actions
    game = rng.integers(0, 2**40, size=m).astype(np.int64)
    decision = rng.integers(0, 40, size=m).astype(np.int32)
    return logits, legal, game, decision


def test_sampler_matches_definition(ext):
    logits, legal, game, decision = _inputs()
    t = lambda a: torch.from_numpy(a).to(DEV)
    actions, logp = ext.sample_actions(t(logits), t(legal), t(game), t(decision), seed_base=12345)
    actions, logp = actions.cpu().numpy(), logp.cpu().numpy()
    noise = gumbel_noise(game, decision, 12345)
    score = np.where(legal, logits[:, :179].astype(np.float64) + noise, -np.inf)
    expect = score.argmax(1)
    srt = np.sort(score, 1)
    clear = (srt[:, -1] - srt[:, -2]) > 1e-4  # float32 vs float64 near-ties excluded
    has = legal.any(1)
    assert actions[5] == -1 and logp[5] == 0.0
    assert (actions[has & clear] == expect[has & clear]).all()
    masked = torch.from_numpy(np.where(legal, logits[:, :179], -1e30).astype(np.float32))
    ref_logp = torch.log_softmax(masked, 1).numpy()[np.arange(len(actions)), np.maximum(actions, 0)]
    assert np.abs(logp[has] - ref_logp[has]).max() < 1e-4


def test_greedy_is_masked_argmax(ext):
    logits, legal, game, decision = _inputs(seed=1)
    t = lambda a: torch.from_numpy(a).to(DEV)
    actions, _ = ext.sample_actions(t(logits), t(legal), t(game), t(decision), greedy=True)
    masked = np.where(legal, logits[:, :179], -np.inf)
    has = legal.any(1)
    assert (actions.cpu().numpy()[has] == masked.argmax(1)[has]).all()
