"""PyTorch restatements of the reference's residual MLP forward (test expectations only).

python/cugo_ppo_nets50.py:26-64 (ResidualBlock/ResidualMlp.forward_hidden), norm="none":
h = inp(x); h = h + fc2(act(fc1(h))) per block; out(act(h)).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def mlp_forward_fp32(weights, biases, x, blocks: int, activation: str) -> torch.Tensor:
    """Exact forward in fp32 from the same bf16 weights and bf16-rounded inputs."""
    act = F.relu if activation == "relu" else F.silu
    w = [t.float() for t in weights]
    b = [t.float() for t in biases]
    x = x.to(torch.bfloat16).float()
    h = F.linear(x, w[0], b[0])
    for i in range(blocks):
        h = h + F.linear(act(F.linear(h, w[1 + 2 * i], b[1 + 2 * i])), w[2 + 2 * i], b[2 + 2 * i])
    return F.linear(act(h), w[-1], b[-1])


def mlp_forward_autocast(weights, biases, x, blocks: int, activation: str) -> torch.Tensor:
    """The reference's forward as it runs in self-play: fp32 modules under bf16
    autocast (python/cugo_ppo50.py:366), on the same (bf16-valued) weights."""
    act = F.relu if activation == "relu" else F.silu
    w = [t.float() for t in weights]
    b = [t.float() for t in biases]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        h = F.linear(x.float(), w[0], b[0])
        for i in range(blocks):
            h = h + F.linear(act(F.linear(h, w[1 + 2 * i], b[1 + 2 * i])), w[2 + 2 * i],
                             b[2 + 2 * i])
        out = F.linear(act(h), w[-1], b[-1])
    return out.float()
