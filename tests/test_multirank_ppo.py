"""CPU: the data-parallel PPO update (cugo_b200/train.py PpoTrainer with world 2 over
gloo).  Ranks whose rollouts hold different numbers of minibatches must still take
the same collective steps: every epoch runs the smallest count, the KL early stop
uses the KL averaged over the ranks, and the averaged gradients keep the networks
identical on every rank.  The returned statistics (losses, entropy, KL, clip
fraction, explained variance) are reduced over the ranks, so every rank reports the
same values for the shared update."""
from __future__ import annotations

import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

ROOT = Path(__file__).resolve().parents[1]
WORLD, MB = 2, 64


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Net(nn.Module):
    """A small fp32 MLP taking the bf16 rows the update feeds its networks."""

    def __init__(self, k: int, n: int, squeeze: bool) -> None:
        super().__init__()
        self.body = nn.Sequential(nn.Linear(k, 32), nn.SiLU(), nn.Linear(32, n))
        self.squeeze = squeeze

    def forward(self, x):
        y = self.body(x.float())
        return y.squeeze(-1) if self.squeeze else y


def _rollout(n: int, seed: int):
    from cugo_b200.train import Rollout
    g = torch.Generator().manual_seed(seed)
    legal = torch.rand((n, 179), generator=g) < 0.1
    legal[torch.arange(n), torch.randint(0, 179, (n,), generator=g)] = True
    actions = torch.multinomial(legal.float(), 1, generator=g).squeeze(1)
    return Rollout(features=torch.rand((n, 720), generator=g).to(torch.bfloat16), legal=legal,
                   actions=actions, logp=torch.full((n,), -2.0),
                   opp_hand=torch.randint(0, 1 << 50, (n,), generator=g),
                   stock=torch.full((n,), -1, dtype=torch.int64),
                   env_ids=torch.arange(n) // 4, seat=torch.arange(n) % 2,
                   returns=torch.randn(n, generator=g), games=n // 4, terminal=n // 4, nagari=0,
                   decision_steps=4, mean_abs_reward0=1.0)


def _rank_main(rank: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from cugo_b200.train import PpoTrainer
        results = []
        for epochs, target_kl in ((2, 0.0), (5, 1e-12)):
            torch.manual_seed(0)  # the same networks on every rank
            actor, critic = _Net(720, 179, False), _Net(770, 1, True)
            trainer = PpoTrainer(actor, critic, lr=1e-3, minibatch=MB, use_graph=False,
                                 world=WORLD)
            # rank 0 holds 5 minibatches, rank 1 holds 3 (and a ragged tail)
            data = _rollout(5 * MB if rank == 0 else 3 * MB + 17, seed=10 + rank)
            stats = trainer.update(data, epochs, entropy_coef=0.01, target_kl=target_kl)
            flat = torch.cat([p.detach().reshape(-1) for p in
                              list(actor.parameters()) + list(critic.parameters())])
            parts = [torch.zeros_like(flat) for _ in range(WORLD)]
            dist.all_gather(parts, flat)
            st = torch.tensor([stats.policy_loss, stats.value_loss, stats.entropy, stats.kl,
                               stats.clipfrac, stats.explained_var], dtype=torch.float64)
            st_parts = [torch.zeros_like(st) for _ in range(WORLD)]
            dist.all_gather(st_parts, st)
            results.append([stats.updates, float((parts[0] - parts[1]).abs().max()),
                            float((flat - _flat_init()).abs().max()),
                            float((st_parts[0] - st_parts[1]).abs().max())])
        np.save(Path(out_dir) / f"rank{rank}.npy", np.array(results, dtype=np.float64))
    finally:
        dist.destroy_process_group()


def _flat_init() -> torch.Tensor:
    torch.manual_seed(0)
    a, c = _Net(720, 179, False), _Net(770, 1, True)
    return torch.cat([p.detach().reshape(-1) for p in list(a.parameters()) + list(c.parameters())])


def test_data_parallel_update_keeps_ranks_in_step():
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_rank_main, args=(_free_port(), tmp), nprocs=WORLD, join=True,
                           start_method="spawn")
        r0, r1 = np.load(Path(tmp) / "rank0.npy"), np.load(Path(tmp) / "rank1.npy")
    # 3 whole minibatches per epoch on both ranks; the early stop at the 8th update on both
    assert r0[0][0] == r1[0][0] == 6
    assert r0[1][0] == r1[1][0] == 8
    for r in (r0, r1):
        assert np.all(r[:, 1] == 0.0)   # identical parameters on the two ranks
        assert np.all(r[:, 2] > 0.0)    # and they did change
        assert np.all(r[:, 3] == 0.0)   # the statistics cover both ranks' rows: equal on each
