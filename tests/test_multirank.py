"""CPU: the multi-GPU host path (cugo_b200/shard.py) with world_size 2 over gloo.

Each rank plays its own seed blocks with the oracle engine (the engine that the GPU
ranks run bit-exactly) and the ranks reduce their statistics; the totals must equal
one process playing the union of the blocks, and the blocks must be disjoint.
"""
from __future__ import annotations

import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cugo_b200.shard import all_reduce, block_start, game_block

ROOT = Path(__file__).resolve().parents[1]
WORLD, STEPS, GAMES = 2, 3, 96


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stats(game0: int, n: int) -> list[float]:
    from oracle import ref
    r = ref.rollout_random(game0, n, threads=1)
    h = np.bitwise_xor.reduce(r["hashes"].astype(np.uint64))
    return [float(n), float(r["decisions"].sum()), float(r["reward0"].sum()),
            float(r["events"].sum()), float(h & np.uint64(0xFFFFFFFF)), float(h >> np.uint64(32))]


def _rank_main(rank: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        totals = [0.0] * 4
        xor_lo, xor_hi = 0, 0
        for s in range(STEPS):
            st = _stats(block_start(s, rank, WORLD, GAMES), GAMES)
            totals = [a + b for a, b in zip(totals, st[:4])]
            xor_lo ^= int(st[4])
            xor_hi ^= int(st[5])
        summed = all_reduce(totals, WORLD, "sum", device="cpu")
        # hash parts are combined on rank 0 after gathering (xor is not a reduce op)
        parts = [torch.zeros(2, dtype=torch.int64) for _ in range(WORLD)]
        dist.all_gather(parts, torch.tensor([xor_lo, xor_hi], dtype=torch.int64))
        slowest = all_reduce([0.25 * (rank + 1)], WORLD, "max", device="cpu")
        if rank == 0:
            lo = hi = 0
            for p in parts:
                lo ^= int(p[0])
                hi ^= int(p[1])
            np.save(Path(out_dir) / "result.npy", np.array(summed + [lo, hi] + slowest, dtype=np.float64))
    finally:
        dist.destroy_process_group()


def _grad_rank_main(rank: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from cugo_b200.ppo import allreduce_gradients
        params = [torch.nn.Parameter(torch.zeros(3, 4)), torch.nn.Parameter(torch.zeros(5))]
        params[0].grad = torch.full((3, 4), float(rank + 1))
        params[1].grad = torch.arange(5, dtype=torch.float32) * (rank + 1)
        allreduce_gradients(params, WORLD)
        if rank == 0:
            np.save(Path(out_dir) / "grads.npy",
                    np.concatenate([params[0].grad.numpy().ravel(), params[1].grad.numpy()]))
    finally:
        dist.destroy_process_group()


def test_gradient_allreduce_averages_over_ranks():
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_grad_rank_main, args=(_free_port(), tmp), nprocs=WORLD, join=True,
                           start_method="spawn")
        got = np.load(Path(tmp) / "grads.npy")
    expect = np.concatenate([np.full(12, 1.5), np.arange(5) * 1.5])
    assert np.allclose(got, expect)


def test_blocks_are_disjoint_and_contiguous():
    seen = torch.cat([game_block(s, r, WORLD, GAMES, "cpu") for s in range(STEPS) for r in range(WORLD)])
    assert torch.equal(seen.sort().values, torch.arange(STEPS * WORLD * GAMES))


@pytest.mark.timeout(300)
def test_two_gloo_ranks_reduce_to_the_single_process_totals(oracle):
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_rank_main, args=(_free_port(), tmp), nprocs=WORLD, join=True,
                           start_method="spawn")
        got = np.load(Path(tmp) / "result.npy")
    ref = _stats(0, STEPS * WORLD * GAMES)
    assert got[:4].tolist() == ref[:4]
    assert int(got[4]) == int(ref[4]) and int(got[5]) == int(ref[5])
    assert got[6] == 0.5  # the maximum over ranks
