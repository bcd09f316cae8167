"""Single-kernel cases of the benchmark (python bench_cases.py CASE DIMS... [--warmup W] [--iters K]).

bench.py imports the multi-kernel cases (ppo, ppoiter, allaction) for its extras;
the ncu summaries under profiles/ were made by running the single-kernel ones.
Each case builds its inputs on the GPU, runs `--warmup` untimed launches, then
times `--iters` launches with CUDA events on the launching stream and prints one
JSON line with the per-launch time and the achieved rate against the algorithmic
bytes or FLOPs of one launch:

  mlp       M H B      the policy forward (B blocks of width H), flops_per_row * M
  gemm      M N K MODE one tcgen05 GEMM layer (MODE plain | silu | residual | pre: the
                       training forward's SiLU layer keeping its pre-activation), 2MNK
  wgrad     R O I      the weight gradient dW = dY^T X over R rows (split-K), 2ROI
  seqwave   [WAVE]     config 4: one wave of sequence-policy self-play (graphed decision
                       steps) under torch.profiler; kernel time per step by kernel
  mlpsample M H B      the self-play policy step: forward and masked Gumbel-max sampling
                       (one fused launch at H = 512), flops_per_row * M
  observe   ROWS       observe_indexed, 3,319 B per row
  step      ROWS       step_indexed on live mid-game rows with random legal actions,
                       521 B per row
  branch    ROOTS PER  branch_indexed, 274 B per branch
  selfplay  SLOTS      the fused config-1 decision kernel, 4,027 B per decision
  attention N R        decode attention with KV append over a [R, 8, 50, 32] bf16 cache,
                       N queries at uniform positions 0..49: (pos + 3) * 1,024 B per query
  allaction R          all-action Q of R mid-game decisions (every legal action branched,
                       3x512 critic) and 4 redealt worlds per decision
  ppoiter   GAMES [H B] one train_ppo50.py iteration at its defaults (3x512 SiLU actor and
                       critic, 2 epochs of 32,768-row minibatches, GAE 0.95)
  refgpu    [GAMES]    the reference's own GPU build (its extension for sm_100 and its
                       Triton decode kernel, staged by baseline/build_ref.py) beside this
                       package's kernels: the torch50_smoke loop, observe/step/branch,
                       decode attention
  ppo       B          one PPO minibatch step (3x512 actor + critic, B rows) on the fused
                       networks, and the same step with plain PyTorch modules under bf16
                       autocast (cuBLAS) for comparison
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

from cugo_b200 import load_extension  # noqa: E402
from cugo_b200.policy import ResidualMlpPolicy  # noqa: E402


def _time(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters / 1e3


def _mid_game(ext, rows: int, decisions: int = 6):
    dev = torch.device("cuda")
    idx = torch.arange(rows, device=dev, dtype=torch.int64)
    states = ext.create(idx + 12345, idx & 1)
    game, dec = idx.clone(), torch.zeros(rows, dtype=torch.int32, device=dev)
    done, steps = torch.zeros_like(dec), torch.zeros(rows, dtype=torch.int64, device=dev)
    feats = torch.empty((rows, 720), dtype=torch.float32, device=dev)
    legal = torch.empty((rows, 179), dtype=torch.bool, device=dev)
    for _ in range(decisions):
        ext.selfplay_random_step(states, game, dec, done, steps, feats, legal)
    return states, feats, legal


def _random_legal(ext, states, ids):
    """A uniformly drawn legal action for each row ids[j] as the row is now (its
    current legal mask, observed here), in the order of ids."""
    legal = ext.observe_indexed(states, ids)[1]
    u = torch.rand(legal.shape, device=legal.device,
                   generator=torch.Generator(device=legal.device).manual_seed(1))
    return torch.where(legal, u, torch.full_like(u, -1.0)).argmax(1)


def seqwave_case(wave: int) -> dict:
    """One wave of config 4 (SeqWaveSelfPlay, one CUDA graph per decision step) after a
    capture wave, its kernels listed by torch.profiler: device time per decision step
    by kernel, largest first, with each kernel's share."""
    from torch.profiler import ProfilerActivity, profile

    from cugo_b200.seq import SeqDecoder
    from cugo_b200.seq_selfplay import SeqWaveSelfPlay
    sp = SeqWaveSelfPlay(SeqDecoder.from_state_dict(SeqDecoder.random_state(0)), wave=wave)
    sp.play_wave(0)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    steps = sp.play_wave(wave)
    b.record()
    torch.cuda.synchronize()
    wave_s = a.elapsed_time(b) / 1e3
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        steps_p = sp.play_wave(2 * wave)
        torch.cuda.synchronize()
    sp.release()
    per = {}
    for ev in prof.key_averages():
        t = getattr(ev, "self_device_time_total", None)
        t = ev.self_cuda_time_total if t is None else t
        if t > 0:
            per[ev.key] = per.get(ev.key, 0.0) + t
    total = sum(per.values())
    top = sorted(per.items(), key=lambda kv: -kv[1])
    return {"wave": wave, "steps": steps, "wave_seconds": wave_s, "ms_per_step": wave_s * 1e3 / steps,
            "games_per_s": wave / wave_s, "profiled_steps": steps_p,
            "kernel_us_per_step": round(total / steps_p, 1),
            "kernels": [{"name": k[:90], "us_per_step": round(v / steps_p, 2),
                         "share": round(v / total, 4)} for k, v in top[:25]]}


def ppo_case(b: int, warmup: int = 3, iters: int = 10) -> dict:
    """One PPO minibatch step (3x512 actor + critic, b rows) on the fused networks,
    eager and CUDA-graphed, and the same step with plain PyTorch modules under bf16
    autocast (cuBLAS), eager and graphed.  FLOPs: 3 x 2 x b x weights (forward,
    data gradient, weight gradient)."""
    from cugo_b200.ppo import (GraphedPpoStep, Minibatch, NativePpoStep, PpoStep, critic_input,
                               fused_actor, fused_critic)
    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(0)
    legal = torch.rand((b, 179), generator=g) < 0.1
    legal[:, 0] = True
    mb = Minibatch(features=torch.rand((b, 720), generator=g).to(dev, torch.bfloat16),
                   legal=legal.to(dev), actions=torch.zeros(b, dtype=torch.int64, device=dev),
                   logp_old=torch.full((b,), -2.0, device=dev),
                   opp_hand=torch.randint(0, 1 << 50, (b,), generator=g).to(dev),
                   adv=torch.randn(b, generator=g).to(dev), ret=torch.randn(b, generator=g).to(dev))
    actor, critic = fused_actor().to(dev), fused_critic().to(dev)
    # The reference trainer's optimizer settings (python/train_ppo50.py:153-156) in
    # every arm.
    opt = torch.optim.Adam(list(actor.parameters()) + list(critic.parameters()), lr=3e-4,
                           eps=1e-5, fused=True, capturable=True)
    step = NativePpoStep(actor, critic, opt)
    sec_eager = _time(lambda: step.step(mb), warmup, iters)
    graphed = GraphedPpoStep(step, mb)
    sec = _time(lambda: graphed(mb), warmup, iters)
    # The same networks on the autograd step (fused GEMMs, torch elementwise and
    # reductions), graphed.
    a2, c2 = fused_actor().to(dev), fused_critic().to(dev)
    opt2 = torch.optim.Adam(list(a2.parameters()) + list(c2.parameters()), lr=3e-4, eps=1e-5,
                            fused=True, capturable=True)
    graphed2 = GraphedPpoStep(PpoStep(a2, c2, opt2), mb)
    sec_autograd = _time(lambda: graphed2(mb), warmup, iters)

    def torch_mlp(inputs, outputs):
        layers = [torch.nn.Linear(inputs, 512)] + [torch.nn.Linear(512, 512) for _ in range(6)]
        layers.append(torch.nn.Linear(512, outputs))
        return torch.nn.ModuleList(layers).to(dev)

    def run_torch(net, x):
        h = net[0](x)
        for i in range(3):
            h = h + net[2 + 2 * i](torch.nn.functional.silu(net[1 + 2 * i](h)))
        return net[-1](torch.nn.functional.silu(h))

    ta, tc = torch_mlp(720, 179), torch_mlp(770, 1)
    topt = torch.optim.Adam(list(ta.parameters()) + list(tc.parameters()), lr=3e-4, eps=1e-5,
                            fused=True, capturable=True)
    cin = critic_input(mb.features, mb.opp_hand)

    def torch_step():
        topt.zero_grad(set_to_none=False)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = run_torch(ta, mb.features.float()).float()
            value = run_torch(tc, cin.float()).float().squeeze(-1)
        lp = torch.log_softmax(logits.masked_fill(~mb.legal, -1.0e30), 1)
        ratio = (lp.gather(1, mb.actions.unsqueeze(1)).squeeze(1) - mb.logp_old).exp()
        pl = -torch.min(ratio * mb.adv, ratio.clamp(0.8, 1.2) * mb.adv).mean()
        ent = -(lp.exp() * lp).sum(1).mean()
        loss = pl - 0.05 * ent + 0.5 * torch.nn.functional.smooth_l1_loss(value, mb.ret)
        loss.backward()
        for grp in (list(ta.parameters()), list(tc.parameters())):
            torch.nn.utils.clip_grad_norm_(grp, 1.0, foreach=True)
        topt.step()

    sec_torch_eager = _time(torch_step, warmup, iters)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            torch_step()
    torch.cuda.current_stream().wait_stream(side)
    tgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(tgraph):
        torch_step()
    sec_torch = _time(tgraph.replay, warmup, iters)
    flops = 3 * 2 * b * sum(p.numel() for n, p in list(actor.named_parameters()) +
                            list(critic.named_parameters()) if n.endswith("weight"))
    return dict(seconds=sec, tflops=flops / sec / 1e12, eager_seconds=sec_eager,
                autograd_step_seconds=sec_autograd,
                torch_autocast_seconds=sec_torch, torch_autocast_tflops=flops / sec_torch / 1e12,
                torch_autocast_eager_seconds=sec_torch_eager,
                speedup_vs_torch_autocast=sec_torch / sec)


def allaction_case(r: int, warmup: int = 3, iters: int = 10) -> dict:
    """All-action values of r mid-game decisions (python/cugo_ppo50.py:87-104) and
    their redealt-world versions (:152-270), timed end to end on the device."""
    from cugo_b200.allaction import action_values, redeal_worlds, world_values
    from cugo_b200.ppo import critic_input, fused_critic
    ext = load_extension()
    dev = torch.device("cuda")
    states, _, legal = _mid_game(ext, r)
    ids = torch.arange(r, device=dev)
    _, legal, players, done, _ = ext.observe_indexed(states, ids)
    keep = torch.nonzero(~done).squeeze(1)
    env_rows, seat, branch = keep, players.index_select(0, keep).long(), legal.index_select(0, keep)
    children = int(branch.sum())
    critic = fused_critic().to(dev)
    scale = 10.0
    with torch.no_grad():
        sec_q = _time(lambda: action_values(ext, critic, states, env_rows, seat, branch, scale),
                      warmup, iters)

        def composed():  # the reference's steps on the same native ops and critic
            rows, acts = torch.nonzero(branch, as_tuple=True)
            child = ext.branch_indexed(states, env_rows.index_select(0, rows), acts)[0]
            cids = torch.arange(child.shape[0], device=dev)
            features, _, mover, _, _ = ext.observe_indexed(child, cids)
            opp = ext.hands_indexed(child, cids).gather(1, (1 - mover.long()).unsqueeze(1)).squeeze(1)
            return critic(critic_input(features, opp))

        sec_ref = _time(composed, warmup, iters)
        rows, acts = torch.nonzero(branch, as_tuple=True)
        child = ext.branch_indexed(states, env_rows.index_select(0, rows), acts)[0]
        cids = torch.arange(child.shape[0], device=dev)
        sec_obs = _time(lambda: ext.observe_critic_bf16(child, cids), warmup, iters)
        sec_redeal = _time(lambda: redeal_worlds(ext, states, env_rows, seat, 4), warmup, iters)
        vs_pool = torch.zeros(seat.shape[0], dtype=torch.bool, device=dev)
        sec_world = _time(lambda: world_values(ext, None, None, states, env_rows, seat, vs_pool,
                                               branch, scale, 4, critic=critic, depth=1),
                          max(1, warmup // 2), max(2, iters // 2))
    return dict(decisions=int(keep.numel()), children=children, action_values_seconds=sec_q,
                children_per_s=children / sec_q, reference_composition_seconds=sec_ref,
                observe_critic_seconds=sec_obs, observe_critic_gbs=children * 1804 / sec_obs / 1e9,
                redeal_worlds4_seconds=sec_redeal, world_values4_seconds=sec_world,
                world_children_per_s=4 * children / sec_world)


def ppoiter_case(games: int, hidden: int = 512, blocks: int = 3, warmup: int = 1,
                 iters: int = 2) -> dict:
    """One PPO iteration (python/train_ppo50.py defaults; hidden/blocks of both
    networks) on the native kernels."""
    from cugo_b200.ppo import fused_actor, fused_critic
    from cugo_b200.train import PpoTrainer, RolloutStorage, iteration
    ext = load_extension()
    dev = torch.device("cuda")
    torch.manual_seed(0)
    actor, critic = fused_actor(hidden, blocks).to(dev), fused_critic(hidden, blocks).to(dev)
    trainer = PpoTrainer(actor, critic)
    storage = RolloutStorage(games * 24, dev)
    for i in range(warmup):
        iteration(ext, trainer, storage, games, 1000 + i)
    runs = [iteration(ext, trainer, storage, games, 2000 + i) for i in range(iters)]
    best = min(runs, key=lambda r: r["seconds"])
    st = best.pop("stats")
    best.update(updates=st.updates, rows_per_s=best["rows"] / best["seconds"],
                games_per_s_collect=games / best["collect_seconds"])
    return best


def _events_time(fn, warmup: int, iters: int, before=None) -> float:
    """Mean seconds of fn() between CUDA events on the current stream; before()
    (e.g. restoring mutated inputs) runs outside each timed launch."""
    for _ in range(warmup):
        if before:
            before()
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        if before:
            before()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        total += a.elapsed_time(b) / 1e3
    return total / iters


def reference_gpu_case(games: int = 262144, warmup: int = 1, iters: int = 2) -> dict:
    """The reference's own GPU build beside this package's kernels, on the same GPU at
    the same shapes: its extension (python/csrc/torch50_ext.cu, built for sm_100 by
    baseline/build_ref.py) and its Triton decode kernel
    (python/cugo_seq_attention50.py:22-40).

      loop      torch50_smoke.run_games (python/torch50_smoke.py:13-59), unchanged, with
                PpoActor(512, 3) in fp16 (as that script runs it; Kaiming-normal weights,
                seed 0) over `games` games, on the reference extension and on this
                package's (the drop-in swap), against play_batch with the 3x512 policy
      observe   observe_indexed on mid-game rows, 3,319 B per row
      step      step_indexed on the same rows (restored before each launch), 521 B/row
      branch    branch_indexed at config 2: 65,536 roots x 256 branches, 274 B/branch
      decode    decode attention, 8,192 queries over an [8,192, 8, 50, 32] bf16 cache:
                the Triton kernel against decode_attention_kernel, and the reference's
                append (index_put_ of k and v) + Triton against the fused append"""
    import time

    from baseline import build_ref
    ref_ext = build_ref.load_reference_extension()
    ref_py = str(build_ref.reference_python())
    if ref_py not in sys.path:
        sys.path.insert(0, ref_py)
    import cugo_ppo_nets50
    import cugo_seq_attention50
    import torch50_smoke

    from cugo_b200.selfplay import play_batch

    ext = load_extension()
    dev = torch.device("cuda")
    out: dict = {"games": games}

    # -- whole loop ------------------------------------------------------------------
    torch.manual_seed(0)
    model = cugo_ppo_nets50.PpoActor(512, 3, norm="none")
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, torch.nn.Linear):
                torch.nn.init.kaiming_normal_(mod.weight)
                torch.nn.init.zeros_(mod.bias)
    model = model.to(dev).half().eval()

    def loop(e, offset):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.inference_mode():
            summary = torch50_smoke.run_games(e, model, games, offset, 128)
        torch.cuda.synchronize()
        return time.perf_counter() - t0, summary

    for name, e in (("reference_ext", ref_ext), ("cugo_ext", ext)):
        for i in range(warmup):
            loop(e, 1_000_000 + i * games)
        runs = [loop(e, 2_000_000 + i * games) for i in range(iters)]
        sec = min(r[0] for r in runs)
        out[f"loop_{name}_games_per_s"] = games / sec
        out[f"loop_{name}_steps"] = runs[0][1]["steps"]
    pol = ResidualMlpPolicy(512, 3, "relu", device=dev, seed=0)
    idx = torch.arange(games, dtype=torch.int64, device=dev)
    for i in range(warmup):
        play_batch(ext, pol, idx + i * games)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(iters):
        play_batch(ext, pol, idx + (warmup + i) * games)
    torch.cuda.synchronize()
    out["play_batch_games_per_s"] = games * iters / (time.perf_counter() - t0)
    out["loop_speedup_same_caller"] = (out["loop_cugo_ext_games_per_s"] /
                                       out["loop_reference_ext_games_per_s"])
    out["loop_speedup_native"] = out["play_batch_games_per_s"] / out["loop_reference_ext_games_per_s"]

    # -- engine ops --------------------------------------------------------------------
    states, _, _ = _mid_game(ext, games)
    ids = torch.randperm(games, device=dev)
    acts = _random_legal(ext, states, ids)
    snapshot = states.clone()
    for name, e in (("reference", ref_ext), ("cugo", ext)):
        sec = _events_time(lambda: e.observe_indexed(states, ids), warmup + 2, iters + 3)
        out[f"observe_{name}_gbs"] = games * 3319 / sec / 1e9
        sec = _events_time(lambda: e.step_indexed(states, ids, acts), warmup + 2, iters + 3,
                           before=lambda: states.copy_(snapshot))
        out[f"step_{name}_gbs"] = games * 521 / sec / 1e9
    roots = ext.branch_roots(65536)
    bids, bacts = ext.branch_actions(roots, 256)
    for name, e in (("reference", ref_ext), ("cugo", ext)):
        sec = _events_time(lambda: e.branch_indexed(roots, bids, bacts), warmup + 1, iters + 1)
        out[f"branch_{name}_per_s"] = bids.numel() / sec
    for k in ("observe", "step"):
        out[f"{k}_speedup"] = out[f"{k}_cugo_gbs"] / out[f"{k}_reference_gbs"]
    out["branch_speedup"] = out["branch_cugo_per_s"] / out["branch_reference_per_s"]

    # -- decode attention ----------------------------------------------------------------
    n = r = 8192
    slots, heads, dh = 50, 8, 32
    g = torch.Generator(device="cpu").manual_seed(0)
    kc = torch.randn((r, heads, slots, dh), generator=g).to(dev, torch.bfloat16)
    vc = torch.randn((r, heads, slots, dh), generator=g).to(dev, torch.bfloat16)
    qkv = torch.randn((n, 3 * heads * dh), generator=g).to(dev, torch.bfloat16)
    pos = torch.randint(0, slots, (n,), generator=g).to(dev)
    rows = torch.randperm(r, generator=g)[:n].to(dev)
    q, kn, vn = (qkv[:, i * 256:(i + 1) * 256].view(n, heads, dh) for i in range(3))
    qc = q.contiguous()
    triton_attn = cugo_seq_attention50.decode_attention
    sec_t = _events_time(lambda: triton_attn(qc, kc, vc, pos, True, rows), warmup + 3, iters + 8)
    sec_o = _events_time(lambda: ext.decode_attention(q, kc, vc, pos, rows), warmup + 3, iters + 8)

    # The reference's append (python/cugo_seq50.py:310-318): index_put_ of the new key
    # and value at (row * heads + head, pos) of the [rows * heads, slots, dh] cache.
    flat_rows = (rows.view(n, 1) * heads + torch.arange(heads, device=dev).view(1, heads)).flatten()
    flat_pos = pos.repeat_interleave(heads)
    kn2, vn2 = kn.reshape(n * heads, dh), vn.reshape(n * heads, dh)

    def ref_append_attend():
        kc.view(-1, slots, dh).index_put_((flat_rows, flat_pos), kn2)
        vc.view(-1, slots, dh).index_put_((flat_rows, flat_pos), vn2)
        return triton_attn(qc, kc, vc, pos, True, rows)

    sec_ta = _events_time(ref_append_attend, warmup + 3, iters + 8)
    sec_oa = _events_time(lambda: ext.decode_attention(q, kc, vc, pos, rows, k_new=kn, v_new=vn),
                          warmup + 3, iters + 8)
    nbytes = int(((pos + 1) * 1024).sum()) + n * 1024
    out.update(decode_triton_us=sec_t * 1e6, decode_cugo_us=sec_o * 1e6,
               decode_triton_gbs=nbytes / sec_t / 1e9, decode_cugo_gbs=nbytes / sec_o / 1e9,
               decode_speedup=sec_t / sec_o, decode_append_reference_us=sec_ta * 1e6,
               decode_append_cugo_us=sec_oa * 1e6, decode_append_speedup=sec_ta / sec_oa)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("dims", nargs="*", type=int)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--mode", default="plain", help="gemm: plain | silu | residual | pre")
    args = ap.parse_args()
    ext = load_extension()
    dev = torch.device("cuda")
    d = args.dims
    out: dict = {"case": args.case, "dims": d}
    if args.case == "mlp":
        m, h, blocks = d
        pol = ResidualMlpPolicy(h, blocks, "relu", device=dev)
        x = torch.randn((m, 720), device=dev).to(torch.bfloat16)
        sec = _time(lambda: pol(x), args.warmup, args.iters)
        out.update(seconds=sec, tflops=pol.flops_per_row() * m / sec / 1e12)
    elif args.case == "gemm":
        m, n, k = d[:3]
        mode = args.mode
        a = torch.randn((m, k), device=dev).to(torch.bfloat16)
        w = (torch.randn((n, k), device=dev) * k ** -0.5).to(torch.bfloat16)
        bias = torch.randn(n, device=dev)
        res = torch.randn((m, n), device=dev).to(torch.bfloat16)
        pre = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        out_t = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        run = {"plain": lambda: ext.linear(a, w, bias, out=out_t),
               "silu": lambda: ext.linear(a, w, bias, out=out_t, act=2),
               "residual": lambda: ext.linear(a, w, bias, residual=res, out=out_t),
               "pre": lambda: ext.linear_pre(a, w, bias, 2, pre, out=out_t)}[mode]
        sec = _time(run, args.warmup, args.iters)
        out.update(mode=mode, seconds=sec, tflops=2 * m * n * k / sec / 1e12)
    elif args.case == "wgrad":
        r, o, i = d
        dy = torch.randn((r, o), device=dev).to(torch.bfloat16)
        x = torch.randn((r, i), device=dev).to(torch.bfloat16)
        dw = torch.empty((o, i), dtype=torch.float32, device=dev)
        sec = _time(lambda: ext.wgrad_bf16(dy, x, dw), args.warmup, args.iters)
        out.update(seconds=sec, tflops=2 * r * o * i / sec / 1e12)
    elif args.case == "seqwave":
        out.update(seqwave_case(d[0] if d else 4096))
    elif args.case == "mlpsample":  # the self-play policy step: MLP + sampling head
        m, h, blocks = d
        pol = ResidualMlpPolicy(h, blocks, "relu", device=dev)
        x = torch.randn((m, 720), device=dev).to(torch.bfloat16)
        bits = ext.pack_legal(torch.rand((m, 179), device=dev) < 0.1)
        game = torch.arange(m, device=dev, dtype=torch.int64)
        dec = torch.zeros(m, dtype=torch.int32, device=dev)
        sec = _time(lambda: pol.forward_sample(x, bits, game, dec), args.warmup, args.iters)
        out.update(seconds=sec, tflops=pol.flops_per_row() * m / sec / 1e12,
                   fused=pol.samples_in_kernel())
    elif args.case == "observe":
        (rows,) = d
        states, _, _ = _mid_game(ext, rows)
        ids = torch.randperm(rows, device=dev)
        sec = _time(lambda: ext.observe_indexed(states, ids), args.warmup, args.iters)
        out.update(seconds=sec, gbs=rows * 3319 / sec / 1e9)
    elif args.case == "step":
        # Live mid-game rows in random order, each given a uniformly drawn legal action
        # of its current decision (the mask observed on the rows as they are now).
        (rows,) = d
        states, _, _ = _mid_game(ext, rows)
        ids = torch.randperm(rows, device=dev)
        acts = _random_legal(ext, states, ids)
        snapshot = states.clone()

        def run():
            states.copy_(snapshot)
            ext.step_indexed(states, ids, acts)

        sec_copy = _time(lambda: states.copy_(snapshot), args.warmup, args.iters)
        sec = _time(run, args.warmup, args.iters) - sec_copy
        out.update(seconds=sec, gbs=rows * 521 / sec / 1e9)
    elif args.case == "branch":
        roots_n, per = d
        roots = ext.branch_roots(roots_n)
        ids, acts = ext.branch_actions(roots, per)
        sec = _time(lambda: ext.branch_indexed(roots, ids, acts), args.warmup, args.iters)
        out.update(seconds=sec, branches_per_s=roots_n * per / sec,
                   gbs=roots_n * per * 274 / sec / 1e9)
    elif args.case == "selfplay":
        (slots,) = d
        idx = torch.arange(slots, device=dev, dtype=torch.int64)
        states = ext.create(idx + 12345, idx & 1)
        game, dec = idx.clone(), torch.zeros(slots, dtype=torch.int32, device=dev)
        done, steps = torch.zeros_like(dec), torch.zeros(slots, dtype=torch.int64, device=dev)
        feats = torch.empty((slots, 720), dtype=torch.float32, device=dev)
        legal = torch.empty((slots, 179), dtype=torch.bool, device=dev)
        acts = torch.empty((slots,), dtype=torch.int64, device=dev)
        sec = _time(lambda: ext.selfplay_random_step(states, game, dec, done, steps, feats, legal,
                                                     actions=acts),
                    args.warmup, args.iters)
        out.update(seconds=sec, decisions_per_s=slots / sec, gbs=slots * 4027 / sec / 1e9)
    elif args.case == "attention":
        n, r = d
        slots, heads, dh = 50, 8, 32
        g = torch.Generator(device="cpu").manual_seed(0)
        kc = torch.randn((r, heads, slots, dh), generator=g).to(dev, torch.bfloat16)
        vc = torch.randn((r, heads, slots, dh), generator=g).to(dev, torch.bfloat16)
        qkv = torch.randn((n, 3 * heads * dh), generator=g).to(dev, torch.bfloat16)
        pos = torch.randint(0, slots, (n,), generator=g).to(dev)
        rows = torch.randperm(r, generator=g)[:n].to(dev)
        q, kn, vn = (qkv[:, i * 256:(i + 1) * 256].view(n, heads, dh) for i in range(3))
        sec = _time(lambda: ext.decode_attention(q, kc, vc, pos, rows, k_new=kn, v_new=vn),
                    args.warmup, args.iters)
        nbytes = int(((pos + 3) * 1024).sum())
        out.update(seconds=sec, gbs=nbytes / sec / 1e9, bytes_per_launch=nbytes)
    elif args.case == "refgpu":
        games = d[0] if d else 262144
        out.update(reference_gpu_case(games, args.warmup, args.iters))
    elif args.case == "allaction":
        (r,) = d
        out.update(allaction_case(r, args.warmup, args.iters))
    elif args.case == "ppoiter":
        games, hidden, blocks = (list(d) + [512, 3])[:3] if len(d) < 3 else d
        out.update(ppoiter_case(games, hidden, blocks, args.warmup, args.iters))
    elif args.case == "ppo":
        (b,) = d
        out.update(ppo_case(b, args.warmup, args.iters))
    else:
        raise SystemExit(f"unknown case {args.case}")
    print(json.dumps(out))


if __name__ == "__main__":
    main()
