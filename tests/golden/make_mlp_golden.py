"""Golden logits from the reference's own PpoActor module (python/cugo_ppo_nets50.py)
imported from the reference tree, on real observations of tests/golden/steps.npz.

    python tests/golden/make_mlp_golden.py      # needs the reference tree

The actor is PpoActor(hidden=64, blocks=2, norm="none") with seeded random weights
(its zero-initialised output layer re-drawn so logits are informative), weights
rounded to bf16 and evaluated in fp32 on bf16-rounded features.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.build import reference_root  # noqa: E402

REF = reference_root() / "python"


def main() -> None:
    sys.path.insert(0, str(REF))
    from cugo_ppo_nets50 import PpoActor  # the reference's module

    torch.manual_seed(0)
    actor = PpoActor(hidden=64, blocks=2, norm="none")
    with torch.no_grad():
        for p in actor.parameters():
            p.normal_(0.0, 0.2)
            p.copy_(p.to(torch.bfloat16).float())
    feats = torch.from_numpy(np.load(HERE / "steps.npz")["features"])
    x = feats.to(torch.bfloat16).float()
    with torch.no_grad():
        logits = actor(x)
    state = {k: v.to(torch.bfloat16).view(torch.int16).numpy() for k, v in actor.state_dict().items()}
    np.savez_compressed(HERE / "ppo_actor_64x2.npz", logits=logits.numpy(), **state)
    print("ppo_actor_64x2.npz", (HERE / "ppo_actor_64x2.npz").stat().st_size)


if __name__ == "__main__":
    main()
