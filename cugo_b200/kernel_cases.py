"""Single-kernel cases for timing and profiling (python -m cugo_b200.kernel_cases CASE ...).

Each case builds its inputs on the GPU, runs `--warmup` untimed launches, then times
`--iters` launches with CUDA events on the launching stream and prints one JSON line
with the per-launch time and the achieved rate against the algorithmic bytes or
FLOPs of one launch:

  gemm      M N K      one tcgen05 layer, 2*M*N*K FLOP
  mlp       M H B      the policy forward (B blocks of width H), flops_per_row * M
  mlpsample M H B      the self-play policy step: forward and masked Gumbel-max sampling
                       (one fused launch at H = 512), flops_per_row * M
  observe   ROWS       observe_indexed, 3,319 B per row
  step      ROWS       step_indexed on live mid-game rows, 521 B per row
  branch    ROOTS PER  branch_indexed, 274 B per branch
  selfplay  SLOTS      the fused config-1 decision kernel, 4,027 B per decision
  sample    ROWS       the Gumbel-max sampler, 180*4 + 179 + 16 B read, 12 B written per row
  attention N R        decode attention with KV append over a [R, 8, 50, 32] bf16 cache,
                       N queries at uniform positions 0..49: (pos + 3) * 1,024 B per query
  seqwave   W WAVES    sequence self-play (4-layer d256 policy), WAVES waves of W games
  seqops    W          each op of one sequence decision step at wave size W, timed alone
  allaction R          all-action Q of R mid-game decisions (every legal action branched,
                       3x512 critic) and 4 redealt worlds per decision: action_values,
                       the reference's composition of the same ops, redeal_worlds,
                       world_values (depth 1), observe_critic_bf16 at 1,804 B per child
  seqgames  S L Q      the sequence training forward over S (game, seat) sequences of L
                       events and Q decisions (4-layer d256 policy): native forward_games
                       and the reference's formulation in PyTorch (bf16 autocast, SDPA
                       with the boolean mask), each timed with CUDA events
  ppoiter   GAMES [H B] one train_ppo50.py iteration at its defaults (3x512 SiLU actor and
                       critic, 2 epochs of 32,768-row minibatches, GAE 0.95): collection
                       with recorded transitions and the update, seconds each
  evaluate  PAIRS      paired evaluation of two 3x512 SiLU actors (2 x PAIRS games to the
                       end): the fused evaluator (one CUDA graph per decision step) and
                       the reference's host-compacting loop over the same ops and networks
  ppo       B          one PPO minibatch step (3x512 actor + critic, B rows) on the fused
                       networks, and the same step with plain PyTorch modules under bf16
                       autocast (cuBLAS) for comparison
"""
from __future__ import annotations

import argparse
import json

import torch

from . import load_extension
from .policy import ResidualMlpPolicy


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


def ppo_case(b: int, warmup: int = 3, iters: int = 10) -> dict:
    """One PPO minibatch step (3x512 actor + critic, b rows) on the fused networks,
    eager and CUDA-graphed, and the same step with plain PyTorch modules under bf16
    autocast (cuBLAS), eager and graphed.  FLOPs: 3 x 2 x b x weights (forward,
    data gradient, weight gradient)."""
    from .ppo import GraphedPpoStep, Minibatch, PpoStep, critic_input, fused_actor, fused_critic
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
    opt = torch.optim.Adam(list(actor.parameters()) + list(critic.parameters()), lr=3e-4,
                           capturable=True)
    step = PpoStep(actor, critic, opt)
    sec_eager = _time(lambda: step.step(mb), warmup, iters)
    graphed = GraphedPpoStep(step, mb)
    sec = _time(lambda: graphed(mb), warmup, iters)

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
    topt = torch.optim.Adam(list(ta.parameters()) + list(tc.parameters()), lr=3e-4,
                            capturable=True)
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
                torch_autocast_seconds=sec_torch, torch_autocast_tflops=flops / sec_torch / 1e12,
                torch_autocast_eager_seconds=sec_torch_eager)


def allaction_case(r: int, warmup: int = 3, iters: int = 10) -> dict:
    """All-action values of r mid-game decisions (python/cugo_ppo50.py:87-104) and
    their redealt-world versions (:152-270), timed end to end on the device."""
    from .allaction import action_values, redeal_worlds, world_values
    from .ppo import critic_input, fused_critic
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


def seqgames_case(s_n: int, length: int, q_n: int, warmup: int = 3, iters: int = 10) -> dict:
    """SeqNet.forward_games (python/cugo_seq50.py:240-265) on the native kernels and, for
    comparison, the same function as the reference formulates it in PyTorch under bf16
    autocast (token embeddings as Linear layers, scaled_dot_product_attention with a
    [S, 1, T, T] boolean mask), on seeded synthetic histories."""
    from types import SimpleNamespace
    from .seq import SeqDecoder
    f = torch.nn.functional
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(0)
    k50 = (1 << 50) - 1
    # Events as the engine writes them: each of the 8 card words holds 0-2 cards.
    cards = torch.randint(0, 50, (s_n, 48, 8, 2), generator=g)
    keep = torch.randint(0, 2, (s_n, 48, 8, 2), generator=g)
    bits = (torch.ones_like(cards) << cards) * keep
    ev = torch.zeros((s_n, 48, 9), dtype=torch.int64)
    ev[..., :8] = bits[..., 0] | bits[..., 1]
    ev[..., 8] = torch.randint(0, 2, (s_n, 48), generator=g) | (torch.randint(0, 12, (s_n, 48), generator=g) << 8)
    count = torch.full((s_n,), length, dtype=torch.int64)
    start = torch.randint(0, 1 << 62, (s_n, 8), generator=g) & k50
    start[:, 6] &= (1 << 12) - 1
    start[:, 7] &= 0xFFFF
    seat = torch.arange(s_n) & 1
    seen = torch.randint(0, length + 1, (s_n, q_n), generator=g).sort(1).values
    feats = torch.rand((s_n, q_n, 720), generator=g).to(torch.bfloat16)
    legal = torch.rand((s_n, q_n, 179), generator=g) < 0.1
    t = {k: v.to(dev) for k, v in dict(events=ev, count=count, start=start, seat=seat, seen=seen,
                                        feats=feats, legal=legal).items()}
    hist = SimpleNamespace(events=t["events"], count=t["count"], start=t["start"], seat=t["seat"])
    state = SeqDecoder.random_state(seed=0)
    dec = SeqDecoder.from_state_dict(state, device=dev)
    p = {k: v.to(dev) for k, v in state.items()}

    def native():
        return dec.forward_games(hist, t["feats"], t["legal"], t["seen"], length=length)

    # The reference's formulation: multi-hot tokens through Linear layers, SDPA with a mask.
    bits = torch.arange(50, device=dev)
    tt = length + 1 + q_n
    allowed = torch.zeros(s_n, tt, tt, dtype=torch.bool, device=dev)
    allowed[:, :, 0] = True
    allowed[:, 1:length + 1, 1:length + 1] = torch.ones(length, length, dtype=torch.bool, device=dev).tril()
    allowed[:, length + 1:, 1:length + 1] = torch.arange(length, device=dev).view(1, 1, -1) < t["seen"].unsqueeze(-1)
    allowed[:, length + 1:, length + 1:] = torch.eye(q_n, dtype=torch.bool, device=dev)
    mask = allowed.unsqueeze(1)

    def lin(x, n):
        return f.linear(x, p[n + ".weight"], p[n + ".bias"])

    def torch_forward():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            e = t["events"][:, :length]
            sv = t["seat"].view(-1, 1)
            mine = (e[..., 8] & 0xFF) == sv
            s0 = sv == 0
            slots = (e[..., 0], torch.where(mine, e[..., 1], 0), e[..., 2],
                     torch.where(s0, e[..., 3], e[..., 4]), torch.where(s0, e[..., 4], e[..., 3]),
                     torch.where(s0, e[..., 5], e[..., 6]), torch.where(s0, e[..., 6], e[..., 5]), e[..., 7])
            planes = [((m.unsqueeze(-1) >> bits) & 1).to(torch.bfloat16) for m in slots]
            kind = f.one_hot(((e[..., 8] >> 8) & 0xFF).clamp_max(11), 12).to(torch.bfloat16)
            drawn = torch.where(mine, 0, ((e[..., 1].unsqueeze(-1) >> bits) & 1).sum(-1))
            tok = torch.cat((*planes, kind, mine.unsqueeze(-1).to(torch.bfloat16),
                             drawn.unsqueeze(-1).to(torch.bfloat16)), -1)
            st = t["start"]
            sp = ((torch.stack((st[:, 0], st[:, 2], st[:, 3], st[:, 4], st[:, 5]), -1).unsqueeze(-1) >> bits) & 1)
            stok = torch.cat((sp.flatten(-2).float(), ((st[:, 6:7] >> bits[:12]) & 1).float(),
                              f.one_hot((st[:, 7] & 0xFF).clamp_max(7), 8).float(),
                              torch.zeros((s_n, 4), device=dev)), -1)
            x = torch.cat(((lin(stok, "start_in") + p["position"][0] + p["token_type"][0]).unsqueeze(1),
                           lin(tok, "event_in") + p["position"][1:length + 1] + p["token_type"][1],
                           lin(f.gelu(lin(torch.cat((t["feats"], t["legal"].to(torch.bfloat16)), -1),
                                          "query_in.0")), "query_in.2") + p["token_type"][2]), 1)
            for i in range(4):
                pre = f"encoder.layers.{i}."
                a = f.layer_norm(x, (256,), p[pre + "norm1.weight"], p[pre + "norm1.bias"])
                qkv = f.linear(a, p[pre + "self_attn.in_proj_weight"], p[pre + "self_attn.in_proj_bias"])
                q, k, v = (z.reshape(s_n, tt, 8, 32).transpose(1, 2) for z in qkv.chunk(3, -1))
                att = f.scaled_dot_product_attention(q, k, v, attn_mask=mask)
                x = x + lin(att.transpose(1, 2).reshape(s_n, tt, 256), pre + "self_attn.out_proj")
                a = f.layer_norm(x, (256,), p[pre + "norm2.weight"], p[pre + "norm2.bias"])
                x = x + lin(f.gelu(lin(a, pre + "linear1")), pre + "linear2")
            h = f.layer_norm(x[:, length + 1:], (256,), p["norm.weight"], p["norm.bias"])
            return lin(f.gelu(lin(h, "head.0")), "head.2").float()

    with torch.no_grad():
        sec = _time(native, warmup, iters)
        sec_torch = _time(torch_forward, warmup, iters)
    rows = s_n * tt
    layer_flops = 2 * rows * (256 * 768 + 256 * 256 + 2 * 256 * 1024) * 4
    query_flops = 2 * s_n * q_n * (899 * 512 + 512 * 256 + 256 * 256 + 256 * 179)
    flops = layer_flops + query_flops
    return dict(sequences=s_n, length=length, queries=q_n, tokens=rows, seconds=sec,
                decisions_per_s=s_n * q_n / sec, tflops=flops / sec / 1e12,
                torch_autocast_seconds=sec_torch, torch_autocast_decisions_per_s=s_n * q_n / sec_torch)


def ppoiter_case(games: int, hidden: int = 512, blocks: int = 3, warmup: int = 1,
                 iters: int = 2) -> dict:
    """One PPO iteration (python/train_ppo50.py defaults; hidden/blocks of both
    networks) on the native kernels."""
    from .ppo import fused_actor, fused_critic
    from .train import PpoTrainer, RolloutStorage, iteration
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


def evaluate_case(pairs: int, warmup: int = 1, iters: int = 3) -> dict:
    """evaluate_paired (python/cugo_eval50.py:137-361): games/s of the fused evaluator
    and of the reference's loop structure (compaction and per-policy index copies every
    step, three host synchronisations per step) on the same native ops and networks."""
    import time
    from .evaluate import evaluate_paired, make_seeds
    from .ppo import FusedResidualMlp
    ext = load_extension()
    dev = torch.device("cuda")
    nets = []
    for seed in (1, 2):
        torch.manual_seed(seed)
        net = FusedResidualMlp(720, 179, 512, 3, "silu").to(dev)
        with torch.no_grad():
            for p in net.parameters():
                p.copy_(torch.randn_like(p) * (1.0 / p.shape[-1]) ** 0.5)
        nets.append(net)
    a, b = nets

    def reference_loop(offset: int) -> float:
        seeds, first = make_seeds(pairs, offset, dev)
        states = ext.create(torch.cat((seeds, seeds)), torch.cat((first, first)))
        a_seat = (torch.arange(2 * pairs, device=dev) >= pairs).long()
        active = torch.arange(2 * pairs, device=dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.no_grad():
            for _ in range(128):
                features, legal, players, done, _ = ext.observe_indexed(states, active)
                keep = torch.nonzero(~done).squeeze(1)
                active, features, legal = active[keep], features[keep], legal[keep]
                if active.numel() == 0:
                    break
                use_a = players[keep].long() == a_seat[active]
                actions = torch.empty(active.numel(), dtype=torch.int64, device=dev)
                for net, rows in ((a, torch.nonzero(use_a).squeeze(1)),
                                  (b, torch.nonzero(~use_a).squeeze(1))):
                    if rows.numel():
                        logits = net(features[rows]).float().masked_fill(~legal[rows], -1.0e30)
                        actions.index_copy_(0, rows, logits.argmax(1))
                _, new_done = ext.step_indexed(states, active, actions)[:2]
                active = active[torch.nonzero(~new_done).squeeze(1)]
                if active.numel() == 0:
                    break
        torch.cuda.synchronize()
        return time.perf_counter() - t0

    for i in range(warmup):
        evaluate_paired(ext, a, b, pairs, 1000 + i, 128)
        reference_loop(1000 + i)
    ours, ref, steps = [], [], 0
    for i in range(iters):
        s = evaluate_paired(ext, a, b, pairs, 2000 + i, 128)
        ours.append(s.seconds)
        steps = s.decision_steps
        ref.append(reference_loop(2000 + i))
    sec, sec_ref = min(ours), min(ref)
    return dict(pairs=pairs, games=2 * pairs, decision_steps=steps, seconds=sec,
                games_per_s=2 * pairs / sec, reference_loop_seconds=sec_ref,
                reference_loop_games_per_s=2 * pairs / sec_ref)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("dims", nargs="*", type=int)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    ext = load_extension()
    dev = torch.device("cuda")
    d = args.dims
    out: dict = {"case": args.case, "dims": d}
    if args.case == "gemm":
        m, n, k = d
        a = torch.randn((m, k), device=dev).to(torch.bfloat16)
        w = (torch.randn((n, k), device=dev) * (2.0 / k) ** 0.5).to(torch.bfloat16)
        b = torch.zeros(n, device=dev, dtype=torch.bfloat16)
        # bf16 rows must be a multiple of 16 bytes; other widths use fp32 rows.
        o = torch.empty((m, n), device=dev, dtype=torch.bfloat16 if n % 8 == 0 else torch.float32)
        sec = _time(lambda: ext.linear(a, w, b, out=o, act=1), args.warmup, args.iters)
        out.update(seconds=sec, tflops=2 * m * n * k / sec / 1e12)
    elif args.case == "mlp":
        m, h, blocks = d
        pol = ResidualMlpPolicy(h, blocks, "relu", device=dev)
        x = torch.randn((m, 720), device=dev).to(torch.bfloat16)
        sec = _time(lambda: pol(x), args.warmup, args.iters)
        out.update(seconds=sec, tflops=pol.flops_per_row() * m / sec / 1e12)
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
        (rows,) = d
        states, _, legal = _mid_game(ext, rows)
        ids = torch.randperm(rows, device=dev)
        acts = legal.to(torch.int64).argmax(1).index_select(0, ids)
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
    elif args.case == "seqwave":
        from .seq import SeqDecoder
        from .seq_selfplay import SeqWaveSelfPlay
        w, waves = d
        sp = SeqWaveSelfPlay(SeqDecoder.from_state_dict(SeqDecoder.random_state(0)), wave=w)
        sp.play_wave(0)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        steps = [sp.play_wave(g * w) for g in range(1, waves + 1)]
        b.record()
        torch.cuda.synchronize()
        sec = a.elapsed_time(b) / 1e3
        out.update(seconds=sec, games_per_s=w * waves / sec, steps=steps)
        sp.release()
    elif args.case == "seqops":
        from .seq import SeqDecoder
        (w,) = d
        dec = SeqDecoder.from_state_dict(SeqDecoder.random_state(0))
        g = torch.Generator(device="cpu").manual_seed(0)
        cache = dec.new_cache(2 * w)
        cache.length.copy_(torch.randint(1, 25, (2 * w,), generator=g).to(dev))
        ops = {}
        for n in (w, 2 * w):
            x = torch.randn((n, 256), generator=g).to(dev)
            a = torch.randn((n, 256), generator=g).to(dev, torch.bfloat16)
            f = torch.randn((n, 1024), generator=g).to(dev, torch.bfloat16)
            L = dec.blocks[0]
            rows = torch.arange(n, device=dev)
            qkv = ext.linear(a, L.w_in, L.b_in)
            q, kn, vn = (qkv[:, i * 256:(i + 1) * 256].view(n, 8, 32) for i in range(3))
            ops[f"layernorm n={n}"] = lambda x=x, L=L: ext.layernorm(x, L.norm1_w, L.norm1_b)
            ops[f"in_proj n={n}"] = lambda a=a, L=L: ext.linear(a, L.w_in, L.b_in)
            ops[f"attention n={n}"] = lambda q=q, kn=kn, vn=vn, rows=rows: ext.decode_attention(
                q, cache.k[0], cache.v[0], cache.length, rows, k_new=kn, v_new=vn, pos_clamp=49)
            ops[f"out_proj n={n}"] = lambda a=a, x=x, L=L: ext.linear(a, L.w_out, L.b_out, residual=x, out=x)
            ops[f"linear1 n={n}"] = lambda a=a, L=L: ext.linear(a, L.w1, L.b1, act=3)
            ops[f"linear2 n={n}"] = lambda f=f, x=x, L=L: ext.linear(f, L.w2, L.b2, residual=x, out=x)
        qin = torch.randn((w, 904), generator=g).to(dev, torch.bfloat16)
        ops["query_token"] = lambda: dec.query_token(qin)
        xr = torch.randn((w, 256), generator=g).to(dev)
        ops["readout"] = lambda: dec.readout(xr)
        # Event words shaped like real ones: one card in each of the first seven
        # masks, none shown, actor and kind in the header word.
        cards = torch.randint(0, 50, (w, 9), generator=g)
        ev = torch.bitwise_left_shift(torch.ones_like(cards), cards)
        ev[:, 7] = 0
        ev[:, 8] = torch.randint(0, 2, (w,), generator=g) | (torch.randint(0, 12, (w,), generator=g) << 8)
        ev = ev.to(dev)
        seats = torch.cat((torch.zeros(w), torch.ones(w))).long().to(dev)
        cnt = torch.randint(0, 40, (w,), generator=g).to(dev)
        ops["event_token n=2w"] = lambda: dec.event_token(ev, seats, cnt)
        res = {}
        for name, fn in ops.items():
            # 20 calls captured in a CUDA graph: the time is the GPU's, not the
            # host's launch rate (as in the graph-captured wave driver).
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(20):
                    fn()
            res[name] = round(_time(graph.replay, args.warmup, args.iters) * 1e6 / 20, 2)
            del graph
        out.update(us=res)
    elif args.case == "allaction":
        (r,) = d
        out.update(allaction_case(r, args.warmup, args.iters))
    elif args.case == "seqgames":
        s_n, length, q_n = d
        out.update(seqgames_case(s_n, length, q_n, args.warmup, args.iters))
    elif args.case == "ppoiter":
        games, hidden, blocks = (list(d) + [512, 3])[:3] if len(d) < 3 else d
        out.update(ppoiter_case(games, hidden, blocks, args.warmup, args.iters))
    elif args.case == "evaluate":
        (p,) = d
        out.update(evaluate_case(p, args.warmup, args.iters))
    elif args.case == "ppo":
        (b,) = d
        out.update(ppo_case(b, args.warmup, args.iters))
    elif args.case == "sample":
        (rows,) = d
        logits = torch.randn((rows, 180), device=dev)
        legal = torch.rand((rows, 179), device=dev) < 0.1
        game = torch.arange(rows, device=dev, dtype=torch.int64)
        dec = torch.zeros(rows, dtype=torch.int32, device=dev)
        sec = _time(lambda: ext.sample_actions(logits, legal, game, dec), args.warmup, args.iters)
        out.update(seconds=sec, gbs=rows * (720 + 179 + 16 + 12) / sec / 1e9)
    else:
        raise SystemExit(f"unknown case {args.case}")
    print(json.dumps(out))


if __name__ == "__main__":
    main()
