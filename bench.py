#!/usr/bin/env python
"""Benchmark of the self-play hot path (prints ONE JSON line on rank 0).

Headline (BASELINE metric): complete games/s of config 3 — PPO self-play with the
3x512 residual MLP policy, 262,144 seeded games per GPU played to settlement
(weak scaling: every rank plays its own disjoint block of deal seeds).  One step
is one such batch: create -> {observe -> policy -> Gumbel-max sample -> step ->
compact} until every game has ended.

Also measured in the same run (inputs resident in HBM, CUDA events):
  engine_only  config 1: 1,048,576 slots x 64 decisions of the fused
               observe -> random-legal pick -> step kernel (auto-reset)
  branching    config 2: 65,536 roots x 256 branches through branch_indexed

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cugo|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import datetime, timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "complete games/s per box (3x512 MLP self-play)"
SEED_BASE = 12345
ARCHS = {"512x3": (512, 3), "2048x4": (2048, 4)}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cugo", "reference"], default="cugo")
    ap.add_argument("--games", type=int, default=262_144, help="games per GPU per step")
    ap.add_argument("--arch", choices=sorted(ARCHS), default="512x3")
    ap.add_argument("--no-extras", action="store_true", help="skip configs 1 and 2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---- distributed plumbing ------------------------------------------------------------

def dist_init(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "cugo":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif args.impl == "cugo":
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def all_reduce(values, world, op="sum"):
    from cugo_b200.shard import all_reduce as _all_reduce
    return _all_reduce(values, world, op, device="cuda")


# ---- clocks ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        # Started before the warm-up: nvidia-smi's start-up queries the driver, and
        # started right at the timed region it slowed the first ~0.2 s of it.
        # Samples are kept for the timed window only (host timestamps).
        self.window: tuple[float, float] | None = None
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])
        target = str(device_index)
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:  # noqa: BLE001 - fall back to the index
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu=timestamp,{self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", target], stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def mark(self, start: float, end: float) -> None:
        """The timed region's host wall-clock window (time.time())."""
        self.window = (start, end)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = [r.split(", ") for r in self.path.read_text().splitlines() if r.count(",") >= 9]
        self.path.unlink(missing_ok=True)

        def stamp(r):
            try:
                return datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                return None

        if self.window is not None:
            lo, hi = self.window
            inside = [r for r in rows if (t := stamp(r)) is not None and lo - 0.05 <= t <= hi + 0.05]
            rows = inside or rows
        rows = [r[1:] for r in rows]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def mlp_traffic(arch: str, policy) -> float | None:
    """DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
    dominant policy kernel on a 262,144-row forward: the fused kernel's, scaled from a
    65,536-row capture by the rows (traffic is the input and output rows); the
    layer-per-launch path's, 4,784 MB over its 8 launches."""
    if arch != "512x3":
        return None
    if policy.samples_in_kernel():
        return FUSED_SAMPLE_TRAFFIC_65536 * 4
    if policy.launches_per_forward() == 1:
        return FUSED_TRAFFIC_65536 * 4
    return 598e6


# ncu DRAM bytes of one fused_mlp_kernel launch on 65,536 rows of the 3x512 policy:
# writing the logits, and with the sampling head (features, legal words, game index
# and decision counter in; action and log p out).
FUSED_TRAFFIC_65536 = 116.3e6
FUSED_SAMPLE_TRAFFIC_65536 = 104.5e6


# ---- config 3: policy self-play --------------------------------------------------------

PREWARM_S = 1.0  # untimed play before the warm-up steps (see selfplay_bench)
REPEATS = 3      # timed regions of K steps per measurement; the median is reported


def selfplay_bench(args, world, rank, ext, policy):
    """Config 3 timed two ways, each over REPEATS regions of exactly K steps,
    interleaved (device-timed region, then end-to-end region, three times) so both
    see the same clocks; the median region of each is reported, the max over ranks
    of each region."""
    from cugo_b200.selfplay import RoundTimer, play_batch
    from cugo_b200.shard import all_gather, game_block

    g = args.games
    dev = torch.device("cuda")
    total_steps = args.warmup + args.steps
    # Game blocks for every step, resident in HBM before timing: rank r, step s
    # plays games (s * world + r) * g .. + g.
    blocks = [game_block(s, rank, world, g, dev) for s in range(total_steps)]
    host_blocks = [b.cpu().pin_memory() for b in blocks[args.warmup:]]
    reward_host = torch.empty(g, dtype=torch.float32).pin_memory()
    clocks = ClockSampler(torch.cuda.current_device())
    time.sleep(0.5)  # let nvidia-smi finish starting before any timing
    # The first ~0.5 s of GPU work in a fresh process runs 5-25% slower on these
    # boards, so the same batch is played for PREWARM_S of wall time before the
    # W warm-up steps.  Nothing from it is kept or counted.
    t_warm = time.perf_counter()
    for _ in range(64):
        play_batch(ext, policy, blocks[0])
        torch.cuda.synchronize()
        if time.perf_counter() - t_warm >= PREWARM_S:
            break
    for s in range(args.warmup):
        play_batch(ext, policy, blocks[s])
    regions = []  # (device seconds, results, launches, e2e wall seconds)
    t_start = time.time()
    for _ in range(REPEATS):
        # Inputs resident in HBM, CUDA events on the launching stream.
        barrier(world)
        launches: list[int] = []
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_dev = time.perf_counter()
        start.record()
        results = []
        for s in range(args.warmup, total_steps):
            r = play_batch(ext, policy, blocks[s], launches=launches)
            results.append((r.games, r.decisions, r.bad_status))
        stop.record()
        barrier(world)
        dev_wall = time.perf_counter() - t_dev
        elapsed = start.elapsed_time(stop) / 1e3
        # End to end through the public API, host wall clock: each step's game
        # indices copied from pinned host memory, its rewards read back.
        barrier(world)
        t0 = time.perf_counter()
        for hb in host_blocks:
            idx = hb.to(dev, non_blocking=True)
            r = play_batch(ext, policy, idx)
            reward_host.copy_(r.reward0, non_blocking=True)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        barrier(world)
        regions.append((elapsed, results, sum(launches), wall, dev_wall))
    clocks.mark(t_start, time.time())
    clk = clocks.stop()
    # The policy's in-loop rate, from CUDA events around every forward of one more
    # (untimed) step: the events' host work is kept out of the timed region.
    timer = RoundTimer(enabled=True)
    play_batch(ext, policy, blocks[args.warmup], timer=timer)
    torch.cuda.synchronize()
    mlp_ms, mlp_launches, mlp_rows = timer.total_ms()

    dev_max = [all_reduce([r[0]], world, op="max")[0] for r in regions]
    e2e_max = [all_reduce([r[3]], world, op="max")[0] for r in regions]
    pick = sorted(range(REPEATS), key=lambda i: dev_max[i])[REPEATS // 2]
    _, results, n_launch, _, _ = regions[pick]
    games = sum(r[0] for r in results)
    decisions = sum(r[1] for r in results)
    bad = sum(r[2] for r in results)
    tot_games, tot_dec, tot_bad = all_reduce([games, decisions, bad], world)
    own_dev = statistics.median(r[0] for r in regions)
    own_e2e = statistics.median(r[3] for r in regions)
    per_rank = [{"rank": i, "ms_per_step": v[0] * 1e3 / args.steps,
                 "e2e_ms_per_step": v[1] * 1e3 / args.steps, "sm_mhz": v[2] if v[2] >= 0 else None,
                 "regions_ms_per_step": [round(x * 1e3 / args.steps, 3) for x in v[3:]]}
                for i, v in enumerate(all_gather(
                    [own_dev, own_e2e, clk["sm_mhz"] if clk["sm_mhz"] is not None else -1.0,
                     *[r[0] for r in regions]], world))]
    return dict(games=tot_games, decisions=tot_dec, bad=tot_bad, elapsed=dev_max[pick],
                mlp_ms=mlp_ms, mlp_launches=mlp_launches, mlp_rows=mlp_rows,
                launches=n_launch, clocks=clk, e2e_elapsed=statistics.median(e2e_max),
                e2e_games=tot_games, h2d=g * 8, d2h=g * 4, per_rank=per_rank,
                regions_s=dev_max, e2e_regions_s=e2e_max,
                dev_wall_regions_s=[all_reduce([r[4]], world, op="max")[0] for r in regions])


# ---- config 1 and 2: engine only -----------------------------------------------------

def engine_only_bench(ext, slots=1 << 20, decisions=64, warm=3):
    dev = torch.device("cuda")
    idx = torch.arange(slots, dtype=torch.int64, device=dev)
    states = ext.create(idx + SEED_BASE, idx & 1)
    slot_game = idx.clone()
    slot_dec = torch.zeros(slots, dtype=torch.int32, device=dev)
    completed = torch.zeros(slots, dtype=torch.int32, device=dev)
    steps = torch.zeros(slots, dtype=torch.int64, device=dev)
    feats = torch.empty((slots, 720), dtype=torch.float32, device=dev)
    legal = torch.empty((slots, 179), dtype=torch.bool, device=dev)
    actions = torch.empty((slots,), dtype=torch.int64, device=dev)
    for _ in range(warm):
        ext.selfplay_random_step(states, slot_game, slot_dec, completed, steps, feats, legal,
                                 actions=actions)
    completed.zero_()
    steps.zero_()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(decisions):
        ext.selfplay_random_step(states, slot_game, slot_dec, completed, steps, feats, legal,
                                 actions=actions)
    b.record()
    torch.cuda.synchronize()
    sec = a.elapsed_time(b) / 1e3
    dec = int(steps.sum())
    games = int(completed.sum())
    return dict(slots=slots, decisions_per_slot=decisions, seconds=sec,
                steps_per_s=dec / sec, games_per_s=games / sec, launches=3 * decisions,
                ms_per_decision_step=sec * 1e3 / decisions, decisions_per_step=dec / decisions)


def branching_bench(ext, roots_n=65_536, per_root=256, reps=3):
    roots = ext.branch_roots(roots_n, seed_base=SEED_BASE)
    ids, actions = ext.branch_actions(roots, per_root, seed_base=SEED_BASE)
    out = ext.branch_indexed(roots, ids, actions)  # warm-up
    del out
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = ext.branch_indexed(roots, ids, actions)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
        del out
    sec = min(times)
    n = roots_n * per_root
    # The children (248 B each) are most of the bytes and are only written: the
    # write-only rate of HBM (torch's fill_ over a buffer of the children's size)
    # is the tighter bound beside the copy rate.
    buf = torch.empty((n * 248,), dtype=torch.uint8, device=roots.device)
    fills = []
    for _ in range(reps + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        buf.fill_(1)
        b.record()
        torch.cuda.synchronize()
        fills.append(a.elapsed_time(b) / 1e3)
    del buf
    return dict(roots=roots_n, branches=n, seconds=sec, branches_per_s=n / sec,
                write_only_gbs=n * 248 / min(fills[1:]) / 1e9)


# ---- config 3 with the 4x2048 policy, config 4: sequence self-play -----------------------

def arch_bench(ext, arch: str, games: int, warmup: int = 1, steps: int = 2) -> dict:
    """Config 3 repeated with another residual-MLP architecture (
    "the same run is repeated with the 4x2048 residual MLP")."""
    from cugo_b200.policy import ResidualMlpPolicy
    from cugo_b200.selfplay import RoundTimer, play_batch

    hidden, blocks = ARCHS[arch]
    policy = ResidualMlpPolicy(hidden, blocks, "relu", device="cuda", seed=0)
    dev = torch.device("cuda")
    for s in range(warmup):
        play_batch(ext, policy, torch.arange(games, dtype=torch.int64, device=dev) + s * games)
    timer = RoundTimer(enabled=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    res = [play_batch(ext, policy, torch.arange(games, dtype=torch.int64, device=dev) + s * games,
                      timer=timer) for s in range(warmup, warmup + steps)]
    b.record()
    torch.cuda.synchronize()
    sec = a.elapsed_time(b) / 1e3
    mlp_ms, _, mlp_rows = timer.total_ms()
    tflops = policy.flops_per_row() * mlp_rows / (mlp_ms / 1e3) / 1e12 if mlp_ms > 0 else 0.0
    return {"arch": arch, "games": games * steps, "seconds": sec,
            "games_per_s": sum(r.games for r in res) / sec,
            "decisions_per_s": sum(r.decisions for r in res) / sec,
            "mlp_tflops": tflops}


def seq_bench(wave: int = 4096, waves: int = 4) -> dict:
    """Config 4: event-sequence policy (4 pre-LN layers, d 256, 8x32 heads, FFN 1024,
    bf16 KV cache) self-play in waves of `wave` games, one CUDA graph per step."""
    from cugo_b200.seq import SeqDecoder
    from cugo_b200.seq_selfplay import SeqWaveSelfPlay

    sp = SeqWaveSelfPlay(SeqDecoder.from_state_dict(SeqDecoder.random_state(0)), wave=wave)
    sp.play_wave(0)  # capture + warm-up
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    steps = [sp.play_wave(g * wave) for g in range(1, waves + 1)]
    b.record()
    torch.cuda.synchronize()
    sec = a.elapsed_time(b) / 1e3
    sp.release()
    return {"wave": wave, "waves": waves, "games": wave * waves, "seconds": sec,
            "games_per_s": wave * waves / sec, "decision_steps_per_wave": steps,
            "policy": "SeqNet hybrid, 4 layers, d 256, 8x32 heads, FFN 1024, random init seed 0"}


# ---- CPU: the reference engine (oracle/_ref) + a PyTorch-CPU policy --------------------

CPU_SAMPLE_GAMES = 16384  # games per CPU sample, in the reference arm and in cpu_baseline


def cpu_actor(arch: str):
    """The reference's own PpoActor class (python/cugo_ppo_nets50.py:26-64, staged
    unmodified by baseline/build_ref.py) in fp32, norm "none", with the weights of
    the GPU arm's policy (Kaiming-normal, seed 0; its 179 logit rows).  Returns the
    module and a description.  Without the staged modules the same layer stack is
    run with torch.nn.functional (and the description says so)."""
    from cugo_b200.policy import ResidualMlpPolicy

    hidden, blocks = ARCHS[arch]
    pol = ResidualMlpPolicy(hidden, blocks, "relu", device="cpu", seed=0)
    ws = [w.float() for w in pol.weights]
    bs = [b.float() for b in pol.biases]
    try:
        from baseline import build_ref
        ref_py = str(build_ref.reference_python())
        if ref_py not in sys.path:
            sys.path.insert(0, ref_py)
        from cugo_ppo_nets50 import PpoActor
    except (ImportError, RuntimeError):
        def forward(x):
            f = torch.nn.functional
            h = f.linear(x, ws[0], bs[0])
            for i in range(blocks):
                h = h + f.linear(f.silu(f.linear(h, ws[1 + 2 * i], bs[1 + 2 * i])), ws[2 + 2 * i],
                                 bs[2 + 2 * i])
            return f.linear(f.silu(h), ws[-1][:179], bs[-1][:179])
        return forward, f"{arch} residual MLP (SiLU, functional restatement of PpoActor)"
    actor = PpoActor(hidden, blocks, norm="none")
    layers = [actor.inp] + [l for b in actor.blocks for l in (b.fc1, b.fc2)] + [actor.out]
    with torch.no_grad():
        for layer, w, b in zip(layers, ws, bs):
            layer.weight.copy_(w[:layer.out_features])
            layer.bias.copy_(b[:layer.out_features])
    return actor.eval(), f"the reference's PpoActor({hidden}, {blocks}) class, fp32"


def cpu_selfplay(games: int, arch: str, threads: int, actor=None) -> dict:
    """Plays `games` seeded games (game i: seed 12345 + i, first player i & 1) to
    settlement on the host: the reference's own engine compiled from its sources
    (oracle/_ref, one shard per thread), the reference PpoActor on PyTorch-CPU and
    masked Gumbel-max sampling with the GPU arm's Philox noise definition (counter
    {game, decision}, oracle/philox_np.py).  Games ended at the deal are settled
    before the first decision, as on the GPU."""
    from oracle import ref
    from oracle.philox_np import gumbel_noise

    torch.set_num_threads(threads)
    if actor is None:
        actor = cpu_actor(arch)[0]
    idx = np.arange(games, dtype=np.int64)
    rows = ref.create(idx + SEED_BASE, idx & 1, threads=threads)
    decision = np.zeros(games, dtype=np.int64)
    t0 = time.perf_counter()
    live = np.ones(games, dtype=bool)
    decisions = 0
    for _ in range(128):
        f, legal, _, done, _ = ref.observe(rows, threads=threads)
        live &= ~done
        if not live.any():
            break
        sel = np.nonzero(live)[0]
        with torch.no_grad():
            logits = actor(torch.from_numpy(f[sel])).numpy()
        noise = gumbel_noise(sel.astype(np.uint64), decision[sel], SEED_BASE)
        score = np.where(legal[sel], logits + noise, -np.inf)
        acts = np.zeros(games, dtype=np.int64)
        acts[sel] = score.argmax(1)
        stepped = ref.step(rows[sel], acts[sel], threads=threads)[0]
        rows[sel] = stepped
        decision[sel] += 1
        decisions += sel.size
    sec = time.perf_counter() - t0
    return dict(games=games, decisions=decisions, seconds=sec, games_per_s=games / sec)


def host_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def workload_config(args, world: int) -> dict:
    """The `config` of both arms' JSON lines (one definition, so they are equal)."""
    return {"workload": f"config3-ppo-selfplay-{args.arch}", "games_per_gpu": args.games,
            "policy": f"{args.arch} residual MLP, 179 logits",
            "parallelism": f"dp{world} (disjoint seed blocks)",
            "l2": "inputs exceed L2 (fp32 features of 262,144 games = 755 MB per round)"}


def reference_arm(args, world, rank):
    if rank != 0:
        return
    threads = host_threads()
    actor, actor_desc = cpu_actor(args.arch)
    for _ in range(args.warmup):
        cpu_selfplay(256, args.arch, threads, actor)
    runs = [cpu_selfplay(CPU_SAMPLE_GAMES, args.arch, threads, actor) for _ in range(args.steps)]
    games = sum(r["games"] for r in runs)
    sec = sum(r["seconds"] for r in runs)
    value = games / sec
    desc = (f"{CPU_SAMPLE_GAMES} seeded games per step played to settlement on {threads} host "
            f"threads: the reference's own engine (include/cugo/**, compiled by oracle/Makefile), "
            f"{actor_desc} on PyTorch-CPU, masked Gumbel-max with Philox noise")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "games/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded deals 12345 + i)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": "games/s", "cores": threads, "kind": "reference",
                         "sample": desc},
        "e2e": {"value": value, "unit": "games/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))


# ---- the data-parallel PPO update (N > 1) ------------------------------------------------

def ppo_dp_bench(world: int, rank: int, rows: int = 32768, warmup: int = 3, iters: int = 10) -> dict:
    """One PPO minibatch step per rank (3x512 SiLU actor + critic, `rows` rows each,
    NativePpoStep with the gradient all-reduce over NCCL: the critic's bucket in
    flight during the actor's backward), and the all-reduce of both buckets alone.
    Device time (CUDA events), max over ranks; every rank takes the same steps."""
    from cugo_b200.ppo import Minibatch, NativePpoStep, fused_actor, fused_critic
    dev = torch.device("cuda")
    torch.manual_seed(0)  # identical networks on every rank
    actor, critic = fused_actor().to(dev), fused_critic().to(dev)
    with torch.no_grad():  # non-zero residual branches and heads
        for p in list(actor.parameters()) + list(critic.parameters()):
            if not p.any():
                p.normal_(0.0, 0.02)
    g = torch.Generator(device="cpu").manual_seed(1 + rank)  # each rank its own shard
    legal = torch.rand((rows, 179), generator=g) < 0.1
    legal[:, 0] = True
    mb = Minibatch(features=torch.rand((rows, 720), generator=g).to(dev, torch.bfloat16),
                   legal=legal.to(dev), actions=torch.zeros(rows, dtype=torch.int64, device=dev),
                   logp_old=torch.full((rows,), -2.0, device=dev),
                   opp_hand=torch.randint(0, 1 << 50, (rows,), generator=g).to(dev),
                   adv=torch.randn(rows, generator=g).to(dev), ret=torch.randn(rows, generator=g).to(dev))
    params = list(actor.parameters()) + list(critic.parameters())
    opt = torch.optim.Adam(params, lr=3e-4, eps=1e-5, fused=True, capturable=True)
    step = NativePpoStep(actor, critic, opt, world=world)

    def timed(fn, n):
        barrier(world)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return all_reduce([a.elapsed_time(b) / 1e3 / n], world, op="max")[0]

    for _ in range(warmup):
        step.step(mb)
    sec_step = timed(lambda: step.step(mb), iters)
    from cugo_b200.ppo import finish_allreduce, start_allreduce
    buckets = [(list(critic.parameters()), step.flat["critic"]),
               (list(actor.parameters()), step.flat["actor"])]
    sec_ar = timed(lambda: [finish_allreduce(start_allreduce(ps, world, f)) for ps, f in buckets], iters)
    # The networks stay identical on every rank (the averaged gradients are).
    total = sum(float(p.detach().double().sum()) for p in params)
    spread = all_reduce([total], world, op="max")[0] - (-all_reduce([-total], world, op="max")[0])
    nbytes = 4 * sum(p.numel() for p in params)
    return {"rows_per_rank": rows, "networks": "3x512 actor + critic (SiLU)", "world": world,
            "step_seconds": sec_step, "rows_per_s": rows * world / sec_step,
            "allreduce_seconds": sec_ar, "bucket_bytes": nbytes,
            "allreduce_busbw_gbs": 2 * (world - 1) / world * nbytes / sec_ar / 1e9,
            "param_sum_spread_over_ranks": spread,
            "note": "eager steps (the graphed step is single-GPU); allreduce_seconds is both "
                    "buckets alone, step_seconds includes them overlapped with the backward"}


# ---- main -------------------------------------------------------------------------------

def main():
    args = parse_args()
    world, rank, local = dist_init(args)
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    from cugo_b200 import load_extension
    from cugo_b200.policy import ResidualMlpPolicy

    ext = load_extension()
    hidden, blocks = ARCHS[args.arch]
    policy = ResidualMlpPolicy(hidden, blocks, "relu", device="cuda", seed=0)
    sp = selfplay_bench(args, world, rank, ext, policy)
    extras = {}
    # Extras and the CPU baseline are single-GPU measurements: at N > 1 every rank
    # would repeat them while all GPUs are held.
    if not args.no_extras and world == 1:
        extras["engine_only"] = engine_only_bench(ext)
        extras["branching"] = branching_bench(ext)
        if args.arch != "2048x4":
            extras["config3_2048x4"] = arch_bench(ext, "2048x4", args.games)
        extras["config4_seq"] = seq_bench()
        from bench_cases import ppo_case
        extras["ppo_update"] = {"minibatch": 32768, "networks": "3x512 actor + critic (SiLU)",
                                **ppo_case(32768, warmup=3, iters=10)}
        from bench_cases import ppoiter_case
        extras["ppo_iteration"] = {"games": 65536, "networks": "3x512 actor + critic (SiLU)",
                                   "epochs": 2, "minibatch": 32768,
                                   **ppoiter_case(65536, 512, 3, warmup=1, iters=1)}
        from bench_cases import allaction_case
        extras["all_action_q"] = {"critic": "3x512 OracleCritic layout (SiLU), every legal action",
                                  **allaction_case(16384, warmup=3, iters=10)}
        from baseline import build_ref
        if build_ref.available():
            from bench_cases import reference_gpu_case
            extras["reference_gpu"] = reference_gpu_case(args.games, warmup=1, iters=2)
        else:
            extras["reference_gpu"] = {"unavailable": "baseline/_ref not staged "
                                                      "(python -m baseline.build_ref)"}
    elif not args.no_extras:
        # The data-parallel update is the one extra with a collective: every rank runs it.
        extras["ppo_update_dp"] = ppo_dp_bench(world, rank)
    peaks = measured_peaks()
    if "engine_only" in extras:
        e = extras["engine_only"]
        # Algorithmic bytes of one decision: observe_indexed 3,319 + mask read 179 +
        # action 8 + step_indexed 521 (ids, action, state read + write, outputs).
        gbs = e["steps_per_s"] * 4027 / 1e9
        e["roofline"] = {"bound": "hbm", "bytes_per_decision": 4027, "achieved": gbs,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"]}
    if "branching" in extras:
        b = extras["branching"]
        gbs = b["branches_per_s"] * 274 / 1e9
        b["roofline"] = {"bound": "hbm", "bytes_per_branch": 274, "achieved": gbs,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                         "write_only_gbs": b["write_only_gbs"],
                         "frac_of_write_only": gbs / b["write_only_gbs"]}
    value = sp["games"] / sp["elapsed"]
    mlp_flops = policy.flops_per_row() * sp["mlp_rows"]
    mlp_tflops = mlp_flops / (sp["mlp_ms"] / 1e3) / 1e12 if sp["mlp_ms"] > 0 else 0.0
    out = {
        "metric": METRIC, "value": value, "unit": "games/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sp["elapsed"] * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded deals (seed 12345 + game), Kaiming-normal bf16 weights (seed 0)",
        "config": workload_config(args, world),
        "timing": {"regions": REPEATS, "reported": "median region (max over ranks) of each kind",
                   "order": "device-timed and end-to-end regions interleaved",
                   "prewarm_s": PREWARM_S, "policy_activation": "relu",
                   "ms_per_step_regions": [round(x * 1e3 / args.steps, 3) for x in sp["regions_s"]],
                   "e2e_ms_per_step_regions": [round(x * 1e3 / args.steps, 3)
                                               for x in sp["e2e_regions_s"]],
                   "device_region_wall_ms_per_step": [round(x * 1e3 / args.steps, 3)
                                                      for x in sp["dev_wall_regions_s"]]},
        "per_rank": sp["per_rank"],
        "decisions_per_s": sp["decisions"] / sp["elapsed"],
        "bad_status": sp["bad"],
        "e2e": {"value": sp["e2e_games"] / sp["e2e_elapsed"], "unit": "games/s",
                "h2d_bytes_per_step": sp["h2d"], "d2h_bytes_per_step": sp["d2h"],
                "clock": "host wall clock (perf_counter) around K steps, synchronised, "
                         "max over ranks"},
        "roofline": {"kernel": ("policy MLP forward + sampling: whole-network CTA-pair kernel "
                                "(fused_mlp_kernel with its sampling head)"
                                if policy.launches_per_forward() == 1 else
                                "policy MLP forward: tcgen05 GEMM layers (gemm_kernel)"),
                     "bound": "tensor",
                     "achieved": mlp_tflops, "peak": peaks["bf16_tflops_sustained"],
                     "unit": "TFLOP/s", "frac": mlp_tflops / peaks["bf16_tflops_sustained"],
                     "traffic": mlp_traffic(args.arch, policy),
                     "traffic_unit": "bytes per launch",
                     "peak_source": peaks["source"] + " (sustained)"},
        "clocks": sp["clocks"],
        "gpu_launches": sp["launches"],
        "extras": extras,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # The reference arm's measurement, repeated here: the same sample size, engine,
        # actor class and noise; three samples (10-20 s of host work).
        threads = host_threads()
        actor, actor_desc = cpu_actor(args.arch)
        cpu_selfplay(256, args.arch, threads, actor)
        runs = [cpu_selfplay(CPU_SAMPLE_GAMES, args.arch, threads, actor) for _ in range(3)]
        sec = sum(r["seconds"] for r in runs)
        out["cpu_baseline"] = {
            "value": 3 * CPU_SAMPLE_GAMES / sec, "unit": "games/s", "cores": threads,
            "kind": "reference", "seconds": sec,
            "sample": f"3 x {CPU_SAMPLE_GAMES} seeded games (12345 + i) to settlement: the "
                      f"reference engine (oracle/_ref), {actor_desc} on PyTorch-CPU, masked "
                      f"Gumbel-max with Philox noise"}
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
