"""CPU: the critic input's planes (cugo_b200.ppo.critic_input) equal the reference's
own card_plane and stock_planes (python/cugo_ppo_nets50.py:104-140), imported from the
staged reference modules (baseline/_ref/python)."""
from __future__ import annotations

import sys

import pytest
import torch

from cugo_b200.ppo import critic_input


def test_critic_input_planes_match_the_reference():
    from baseline import build_ref
    try:
        path = str(build_ref.reference_python())
    except RuntimeError as e:
        pytest.skip(str(e))
    if path not in sys.path:
        sys.path.insert(0, path)
    from cugo_ppo_nets50 import card_plane, stock_planes
    g = torch.Generator().manual_seed(0)
    n = 500
    features = torch.randn((n, 720), generator=g).to(torch.bfloat16)
    opp = torch.randint(0, 1 << 50, (n,), generator=g)
    cards = torch.randint(0, 50, (n, 8), generator=g)
    cards[::7, 5:] = 0xFF  # fewer than 8 standard draws left
    stock = sum(cards[:, k] << (8 * k) for k in range(8))
    expect = torch.cat((features, card_plane(opp, torch.bfloat16), stock_planes(stock, torch.bfloat16)), 1)
    assert torch.equal(critic_input(features, opp, stock), expect)
    assert torch.equal(critic_input(features, opp), expect[:, :770])
