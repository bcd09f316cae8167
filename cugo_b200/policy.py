"""Residual-MLP policy/value network of the self-play path.

Architecture (reference python/cugo_ppo_nets50.py:26-64, ResidualMlp/PpoActor with
norm="none"):  h = W_in x + b;  h = h + W2 act(W1 h + b1) + b2  (per block);
out = W_out act(h) + b_out.  The reference uses SiLU; the benchmark configuration
(config 3) uses ReLU and appends a scalar value output to the 179 policy logits.
Weights are bf16 with fp32 accumulation, as under the reference's bf16 autocast
(python/cugo_ppo50.py:366).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

FEATURES = 720
ACTIONS = 179


class ResidualMlpPolicy:
    def __init__(self, hidden: int = 512, blocks: int = 3, activation: str = "relu",
                 outputs: int = ACTIONS + 1, device: torch.device | str = "cuda",
                 seed: int | None = 0) -> None:
        if activation not in ("relu", "silu"):
            raise ValueError("activation must be relu or silu")
        self.hidden, self.blocks, self.activation, self.outputs = hidden, blocks, activation, outputs
        self.device = torch.device(device)
        shapes = [(hidden, FEATURES)] + [(hidden, hidden)] * (2 * blocks) + [(outputs, hidden)]
        gen = torch.Generator().manual_seed(seed if seed is not None else 0)
        self.weights: list[torch.Tensor] = []
        self.biases: list[torch.Tensor] = []
        for shape in shapes:
            w = torch.empty(shape, dtype=torch.float32)
            # Kaiming-normal (fan_in, gain sqrt(2)), drawn on the CPU generator.
            std = (2.0 / shape[1]) ** 0.5
            w.normal_(0.0, std, generator=gen)
            self.weights.append(w.to(self.device, torch.bfloat16).contiguous())
            self.biases.append(torch.zeros(shape[0], dtype=torch.bfloat16, device=self.device))

    @classmethod
    def from_state_dict(cls, state: dict[str, torch.Tensor], blocks: int, activation: str = "silu",
                        device: torch.device | str = "cuda") -> "ResidualMlpPolicy":
        """Loads a reference ResidualMlp/PpoActor state dict (inp, blocks.i.fc1/fc2, out)."""
        hidden = state["inp.weight"].shape[0]
        outputs = state["out.weight"].shape[0]
        self = cls(hidden, blocks, activation, outputs, device, seed=None)
        names = ["inp"] + [f"blocks.{i}.fc{j}" for i in range(blocks) for j in (1, 2)] + ["out"]
        for k, name in enumerate(names):
            self.weights[k] = state[f"{name}.weight"].to(self.device, torch.bfloat16).contiguous()
            self.biases[k] = state[f"{name}.bias"].to(self.device, torch.bfloat16).contiguous()
        return self

    def flops_per_row(self) -> int:
        return 2 * sum(w.shape[0] * w.shape[1] for w in self.weights)

    def _act(self, x: torch.Tensor) -> torch.Tensor:
        return F.relu(x) if self.activation == "relu" else F.silu(x)

    @torch.no_grad()
    def forward(self, features: torch.Tensor) -> torch.Tensor:
        """fp32 [M, 720] features -> fp32 [M, outputs] logits (and value)."""
        x = features.to(torch.bfloat16)
        w, b = self.weights, self.biases
        h = F.linear(x, w[0], b[0])
        for i in range(self.blocks):
            h = h + F.linear(self._act(F.linear(h, w[1 + 2 * i], b[1 + 2 * i])), w[2 + 2 * i],
                             b[2 + 2 * i])
        return F.linear(self._act(h), w[-1], b[-1]).float()

    __call__ = forward
