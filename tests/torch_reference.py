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


class TorchResidualMlp(torch.nn.Module):
    """The reference's ResidualMlp with norm="none" in plain PyTorch (fp32 modules;
    run it under bf16 autocast for the reference's training numerics), with the
    same parameter names (inp, blocks.i.fc1/fc2, out)."""

    def __init__(self, inputs: int, outputs: int, hidden: int, blocks: int,
                 activation: str = "silu") -> None:
        super().__init__()
        self.act = F.relu if activation == "relu" else F.silu
        self.inp = torch.nn.Linear(inputs, hidden)
        self.blocks = torch.nn.ModuleList(
            torch.nn.ModuleDict({"fc1": torch.nn.Linear(hidden, hidden),
                                 "fc2": torch.nn.Linear(hidden, hidden)}) for _ in range(blocks))
        self.out = torch.nn.Linear(hidden, outputs)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.inp(x)
        for b in self.blocks:
            h = h + b["fc2"](self.act(b["fc1"](h)))
        return self.out(self.act(h))


def ppo_losses_reference(logits, value, legal, actions, logp_old, adv, ret, clip: float):
    """The plain-target PPO losses of python/cugo_ppo50.py:572-603 (restated)."""
    log_probs = torch.log_softmax(logits.float().masked_fill(~legal, -1.0e30), dim=1)
    new_logp = log_probs.gather(1, actions.unsqueeze(1)).squeeze(1)
    ratio = (new_logp - logp_old).exp()
    plain = -torch.min(ratio * adv, ratio.clamp(1 - clip, 1 + clip) * adv)
    entropy = -(log_probs.exp() * log_probs).sum(dim=1).mean()
    value_loss = F.smooth_l1_loss(value.float(), ret)
    return plain.mean(), value_loss, entropy
