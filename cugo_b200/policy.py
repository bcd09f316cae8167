"""Residual-MLP policy/value network of the self-play path, on tcgen05 tensor cores.

Architecture (reference python/cugo_ppo_nets50.py:26-64, ResidualMlp/PpoActor with
norm="none"):  h = W_in x + b;  h = h + W2 act(W1 h + b1) + b2  (per block);
out = W_out act(h) + b_out.  The reference uses SiLU; the benchmark configuration
(config 3) uses ReLU and appends a scalar value output to the 179 policy logits.
Weights are bf16 with fp32 accumulation, as under the reference's bf16 autocast
(python/cugo_ppo50.py:366).  Every layer is one launch of the tcgen05 GEMM
(cugo_b200_gemm_bf16) with bias, activation and the residual add in its epilogue,
the last block writing act(h) for the head; at hidden 512 the whole network can
instead run as one launch of the fused MLP kernel (cugo_b200_mlp_fused: a 128-row
tile's activations stay in shared and tensor memory from the input layer to the
head), selected by fused_mlp_supported.
"""
from __future__ import annotations

import os

import torch

FEATURES = 720
ACTIONS = 179
_ACT = {"none": 0, "relu": 1, "silu": 2}


# Whether hidden-512 networks run on the whole-network kernel when the environment
# does not say (CUGO_B200_MLP_FUSED=1 selects it, =0 the layer-per-launch path).
FUSED_MLP_DEFAULT = True


def fused_mlp_supported(hidden: int, blocks: int, inputs: int, outputs: int) -> bool:
    """Whether the whole-network kernel (cugo_b200_mlp_fused) runs this shape: hidden
    512, at most 4 blocks, inputs a multiple of 8 up to 1,024, at most 256 outputs,
    and it is selected (CUGO_B200_MLP_FUSED, else FUSED_MLP_DEFAULT)."""
    env = os.environ.get("CUGO_B200_MLP_FUSED")
    wanted = FUSED_MLP_DEFAULT if env is None else env == "1"
    return (wanted and hidden == 512 and blocks <= 4 and inputs % 8 == 0 and inputs <= 1024
            and outputs <= 256)


class ResidualMlpPolicy:
    def __init__(self, hidden: int = 512, blocks: int = 3, activation: str = "relu",
                 outputs: int = ACTIONS + 1, device: torch.device | str = "cuda",
                 seed: int | None = 0, inputs: int = FEATURES) -> None:
        if activation not in ("relu", "silu"):
            raise ValueError("activation must be relu or silu")
        self.hidden, self.blocks, self.activation, self.outputs = hidden, blocks, activation, outputs
        self.inputs = inputs
        self.device = torch.device(device)
        shapes = [(hidden, inputs)] + [(hidden, hidden)] * (2 * blocks) + [(outputs, hidden)]
        gen = torch.Generator().manual_seed(seed if seed is not None else 0)
        self.weights: list[torch.Tensor] = []
        self.biases: list[torch.Tensor] = []
        for shape in shapes:
            w = torch.empty(shape, dtype=torch.float32)
            # Kaiming-normal (fan_in, gain sqrt(2)), drawn on the CPU generator.
            w.normal_(0.0, (2.0 / shape[1]) ** 0.5, generator=gen)
            self.weights.append(w.to(self.device, torch.bfloat16).contiguous())
            self.biases.append(torch.zeros(shape[0], dtype=torch.bfloat16, device=self.device))
        self._ext = None
        self.error = (torch.zeros(1, dtype=torch.int32, device=self.device)
                      if self.device.type == "cuda" else None)

    @classmethod
    def from_state_dict(cls, state: dict[str, torch.Tensor], blocks: int, activation: str = "silu",
                        device: torch.device | str = "cuda") -> "ResidualMlpPolicy":
        """Loads a reference ResidualMlp/PpoActor/OracleCritic state dict
        (inp, blocks.i.fc1/fc2, out), e.g. from a train_ppo50.py checkpoint."""
        if any(k.endswith("norm.weight") for k in state):
            raise ValueError("ResidualMlpPolicy runs norm='none' networks; load a LayerNorm "
                             "network as cugo_b200.ppo.FusedResidualMlp(..., norm='layer')")
        hidden, inputs = state["inp.weight"].shape
        outputs = state["out.weight"].shape[0]
        self = cls(hidden, blocks, activation, outputs, device, seed=None, inputs=inputs)
        names = ["inp"] + [f"blocks.{i}.fc{j}" for i in range(blocks) for j in (1, 2)] + ["out"]
        for k, name in enumerate(names):
            self.weights[k] = state[f"{name}.weight"].to(self.device, torch.bfloat16).contiguous()
            self.biases[k] = state[f"{name}.bias"].to(self.device, torch.bfloat16).contiguous()
        return self

    def flops_per_row(self) -> int:
        return 2 * sum(w.shape[0] * w.shape[1] for w in self.weights)

    def launches_per_step(self) -> int:
        """Kernel launches of forward_sample (the policy and the sampler)."""
        return 1 if self.samples_in_kernel() else self.launches_per_forward() + 1

    def launches_per_forward(self) -> int:
        if fused_mlp_supported(self.hidden, self.blocks, self.inputs, self.outputs):
            return 1
        return 2 + 2 * self.blocks

    def _extension(self):
        if self._ext is None:
            from .ext import load_extension
            self._ext = load_extension()
        return self._ext

    def _fp32_biases(self) -> list[torch.Tensor]:
        key = tuple((b.data_ptr(), b._version) for b in self.biases)
        if getattr(self, "_bkey", None) != key:
            self._b32 = [b.float().contiguous() for b in self.biases]
            self._bkey = key
        return self._b32

    @torch.no_grad()
    def forward(self, features: torch.Tensor) -> torch.Tensor:
        """[M, inputs] features (bf16, or fp32 cast to bf16 as autocast does) ->
        fp32 [M, outputs] logits (and value)."""
        ext = self._extension()
        x = features if features.dtype == torch.bfloat16 else features.to(torch.bfloat16)
        x = x.contiguous()
        m = x.size(0)
        act = _ACT[self.activation]
        w, b = self.weights, self.biases
        if fused_mlp_supported(self.hidden, self.blocks, self.inputs, self.outputs):
            return ext.mlp_fused(x, w, self._fp32_biases(), act, error=self.error)
        h = torch.empty((m, self.hidden), dtype=torch.bfloat16, device=x.device)
        ext.linear(x, w[0], b[0], out=h, act_after=act if self.blocks == 0 else 0, error=self.error)
        if self.blocks:
            u = torch.empty_like(h)
            for i in range(self.blocks):
                ext.linear(h, w[1 + 2 * i], b[1 + 2 * i], out=u, act=act, error=self.error)
                ext.linear(u, w[2 + 2 * i], b[2 + 2 * i], residual=h, out=h,
                           act_after=act if i == self.blocks - 1 else 0, error=self.error)
        # fp32 rows padded to a multiple of 16 bytes for the vector stores.
        padded = (self.outputs + 3) // 4 * 4
        out = torch.empty((m, padded), dtype=torch.float32, device=x.device)[:, :self.outputs]
        ext.linear(h, w[-1], b[-1], out=out, error=self.error)
        return out

    __call__ = forward

    def samples_in_kernel(self) -> bool:
        """Whether forward_sample runs as one fused kernel (and takes bit-word masks)."""
        return fused_mlp_supported(self.hidden, self.blocks, self.inputs, self.outputs) \
            and self.outputs >= ACTIONS

    @torch.no_grad()
    def forward_sample(self, features: torch.Tensor, legal: torch.Tensor, game: torch.Tensor,
                       decision: torch.Tensor, seed_base: int = 12345, greedy: bool = False,
                       m_dev: torch.Tensor | None = None, rows: torch.Tensor | None = None):
        """Actions and log-probabilities of the masked Gumbel-max sampler over this
        policy's logits (cugo_b200_sample_actions' definition): in the fused MLP's
        head when it runs this shape, else the forward followed by the sampler.
        legal: bool [m, 179], or (fused head only) its int64 [m, 3] bit words; m_dev
        (fused head only): a device-resident row count, rows past it are skipped; rows:
        row r's game and decision are game[rows[r]], decision[rows[r]]."""
        ext = self._extension()
        x = features if features.dtype == torch.bfloat16 else features.to(torch.bfloat16)
        x = x.contiguous()
        if self.samples_in_kernel():
            actions, logp, _ = ext.mlp_fused_sample(x, self.weights, self._fp32_biases(),
                                                    _ACT[self.activation], legal, game, decision,
                                                    seed_base, greedy, m_dev=m_dev, rows=rows)
            return actions, logp
        if m_dev is not None:
            raise RuntimeError("a device-resident row count needs the fused policy step")
        if rows is not None:
            game, decision = game.index_select(0, rows), decision.index_select(0, rows)
        return ext.sample_actions(self.forward(x), legal, game, decision, seed_base, greedy=greedy)
