"""GPU: the whole-network MLP kernel (cugo_b200_mlp_fused) against the fp32 forward of
the same bf16 weights (python/cugo_ppo_nets50.py:26-64, norm "none") and the
layer-per-launch path.

Tolerance: the error against the exact fp32 forward is no larger than 1.25x that of
the reference's own bf16-autocast forward (+1e-3), at most 1e-2 of the output scale;
the argmax agrees wherever the top-2 margin exceeds 4x the error.
"""
from __future__ import annotations

import pytest
import torch

from tests.torch_reference import mlp_forward_autocast, mlp_forward_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
ACT = {"relu": 1, "silu": 2}


def _net(k_in, blocks, n_out, seed):
    g = torch.Generator().manual_seed(seed)
    shapes = [(512, k_in)] + [(512, 512)] * (2 * blocks) + [(n_out, 512)]
    ws = [(torch.randn(s, generator=g) * (2.0 / s[1]) ** 0.5).to(DEV, torch.bfloat16) for s in shapes]
    bs = [(torch.randn(s[0], generator=g) * 0.05).to(DEV) for s in shapes]
    return ws, bs


@pytest.mark.parametrize("m,k_in,blocks,n_out,act", [
    (1000, 720, 3, 180, "relu"), (129, 720, 3, 179, "silu"), (70000, 720, 3, 180, "relu"),
    (300, 512, 0, 64, "relu"), (1000, 1024, 4, 256, "silu"), (1, 720, 1, 1, "relu"),
    (4099, 776, 3, 1, "silu"), (257, 8, 2, 16, "relu"), (2000, 720, 4, 180, "relu")])
def test_fused_mlp_matches_fp32(ext, m, k_in, blocks, n_out, act):
    ws, bs = _net(k_in, blocks, n_out, seed=m + k_in)
    g = torch.Generator().manual_seed(1)
    x = torch.rand((m, k_in), generator=g).to(DEV, torch.bfloat16)
    err_flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ext.mlp_fused(x, ws, bs, ACT[act], error=err_flag)
    torch.cuda.synchronize()
    assert int(err_flag) == 0
    assert out.shape == (m, n_out)
    exact = mlp_forward_fp32(ws, bs, x, blocks, act)
    auto = mlp_forward_autocast(ws, bs, x, blocks, act)
    scale = max(1.0, float(exact.abs().max()))
    err = float((out - exact).abs().max())
    err_ref = float((auto - exact).abs().max())
    assert err <= 1.25 * err_ref + 1e-3, (err, err_ref)
    assert err <= 1e-2 * scale, (err, scale)
    if n_out > 1:
        top2 = exact.topk(2, dim=1).values
        clear = (top2[:, 0] - top2[:, 1]) > 4 * err
        assert torch.equal(out.argmax(1)[clear], exact.argmax(1)[clear])


def test_fused_mlp_without_some_biases(ext):
    # Layers without a bias read zeros, from the shared-memory copy (layers 0..7) and
    # from the global path (layer 8 of a four-block network) alike.
    ws, bs = _net(720, 4, 180, seed=11)
    keep = [b if i % 3 else None for i, b in enumerate(bs)]
    zeros = [b if b is not None else torch.zeros(w.shape[0], device=DEV) for b, w in zip(keep, ws)]
    g = torch.Generator().manual_seed(5)
    x = torch.rand((3000, 720), generator=g).to(DEV, torch.bfloat16)
    out = ext.mlp_fused(x, ws, keep, ACT["relu"])
    ref = ext.mlp_fused(x, ws, zeros, ACT["relu"])
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    exact = mlp_forward_fp32(ws, zeros, x, 4, "relu")
    assert float((out - exact).abs().max()) <= 1e-2 * max(1.0, float(exact.abs().max()))


def test_fused_mlp_is_deterministic_and_respects_strides(ext):
    ws, bs = _net(720, 3, 180, seed=3)
    g = torch.Generator().manual_seed(2)
    big = torch.rand((3000, 728), generator=g).to(DEV, torch.bfloat16)
    x = big[:, :720]  # row stride 728
    out = torch.full((3000, 184), 7.0, device=DEV)
    ext.mlp_fused(x, ws, bs, 1, out=out[:, :180])
    again = ext.mlp_fused(x.contiguous(), ws, bs, 1)
    assert torch.equal(out[:, :180], again)
    assert bool((out[:, 180:] == 7.0).all())
    nob = ext.mlp_fused(x, ws, [None] * len(ws), 1)
    exact = mlp_forward_fp32(ws, [torch.zeros_like(b) for b in bs], x, 3, "relu")
    assert float((nob - exact).abs().max()) <= 1e-2 * max(1.0, float(exact.abs().max()))


def test_policy_routes_through_the_fused_kernel(ext, monkeypatch):
    from cugo_b200.policy import ResidualMlpPolicy
    pol = ResidualMlpPolicy(512, 3, "relu", device=DEV, seed=0)
    monkeypatch.setenv("CUGO_B200_MLP_FUSED", "1")
    assert pol.launches_per_forward() == 1
    g = torch.Generator().manual_seed(4)
    x = torch.rand((5000, 720), generator=g).to(DEV)
    fused = pol(x)
    monkeypatch.setenv("CUGO_B200_MLP_FUSED", "0")
    assert pol.launches_per_forward() == 8
    layers = pol(x)
    exact = mlp_forward_fp32(pol.weights, pol.biases, x, 3, "relu")
    scale = max(1.0, float(exact.abs().max()))
    assert float((fused - layers).abs().max()) <= 1e-2 * scale
    assert float((fused - exact).abs().max()) <= 1e-2 * scale


@pytest.mark.parametrize("m,n_out,greedy,density", [(70000, 180, False, 0.1), (1000, 179, True, 0.3),
                                                   (333, 256, False, 0.02), (129, 180, False, 0.0)])
def test_fused_sampling_head_matches_the_sampler(ext, m, n_out, greedy, density):
    """Actions equal cugo_b200_sample_actions on the kernel's own logits (same noise,
    same tie rule); log p within 1e-5 (the log-sum-exp adds in another order)."""
    ws, bs = _net(720, 3, n_out, seed=m)
    g = torch.Generator().manual_seed(7)
    x = torch.rand((m, 720), generator=g).to(DEV, torch.bfloat16)
    legal = torch.rand((m, 179), generator=g) < density
    legal[::7, :] = False  # rows without a legal action: -1, log p 0
    legal[1::7, 5] = True
    legal = legal.to(DEV)
    game = torch.randint(0, 1 << 40, (m,), generator=g).to(DEV)
    decision = torch.randint(0, 60, (m,), generator=g, dtype=torch.int32).to(DEV)
    actions, logp, logits = ext.mlp_fused_sample(x, ws, bs, 2, legal, game, decision, seed_base=99,
                                                 greedy=greedy, want_logits=True)
    assert torch.equal(logits, ext.mlp_fused(x, ws, bs, 2))
    ref_a, ref_lp = ext.sample_actions(logits.contiguous() if n_out % 4 else logits, legal, game,
                                       decision, seed_base=99, greedy=greedy)
    assert torch.equal(actions, ref_a)
    assert float((logp - ref_lp).abs().max()) <= 1e-5 * max(1.0, float(ref_lp.abs().max()))
    assert bool((actions[::7] == -1).all()) and bool((logp[::7] == 0).all())
    a2, lp2, none = ext.mlp_fused_sample(x, ws, bs, 2, legal, game, decision, seed_base=99,
                                         greedy=greedy)
    assert none is None and torch.equal(a2, actions) and torch.equal(lp2, logp)


def test_fused_sampling_head_reads_game_and_decision_through_rows(ext):
    """rows[r] selects row r's game index and decision counter; an entry outside the
    arrays samples nothing (-1, log p 0)."""
    ws, bs = _net(720, 3, 180, seed=21)
    g = torch.Generator().manual_seed(8)
    m, n_games = 3000, 5000
    x = torch.rand((m, 720), generator=g).to(DEV, torch.bfloat16)
    legal = (torch.rand((m, 179), generator=g) < 0.1).to(DEV)
    game = torch.randint(0, 1 << 40, (n_games,), generator=g).to(DEV)
    decision = torch.randint(0, 60, (n_games,), generator=g, dtype=torch.int32).to(DEV)
    rows = torch.randperm(n_games, generator=g)[:m].to(DEV)
    rows[5], rows[6] = -1, n_games  # outside the arrays
    a, lp, _ = ext.mlp_fused_sample(x, ws, bs, 1, legal, game, decision, seed_base=7, rows=rows)
    safe = rows.clamp(0, n_games - 1)
    ra, rlp, _ = ext.mlp_fused_sample(x, ws, bs, 1, legal, game.index_select(0, safe),
                                      decision.index_select(0, safe), seed_base=7)
    ok = torch.ones(m, dtype=torch.bool, device=DEV)
    ok[5:7] = False
    assert torch.equal(a[ok], ra[ok]) and torch.equal(lp[ok], rlp[ok])
    assert bool((a[~ok] == -1).all()) and bool((lp[~ok] == 0).all())
    with pytest.raises(RuntimeError):
        ext.mlp_fused_sample(x, ws, bs, 1, legal, game, decision, rows=rows[:10])


def test_observe_bits_and_pack_legal_agree_with_the_bool_mask(ext):
    idx = torch.arange(5000, device=DEV, dtype=torch.int64)
    states = ext.create(idx + 31, idx & 1)
    ids = torch.randint(0, 5000, (7777,), device=DEV)
    ids[3] = 9999  # out of range: an empty mask
    f, legal, p, d, st = ext.observe_indexed_bf16(states, ids)
    f2, bits, p2, d2, st2 = ext.observe_indexed_bf16_bits(states, ids)
    assert torch.equal(f, f2) and torch.equal(p, p2) and torch.equal(d, d2) and torch.equal(st, st2)
    assert torch.equal(bits, ext.pack_legal(legal))
    a = torch.arange(179, device=DEV)
    words = bits.gather(1, (a // 64).expand(bits.shape[0], -1))
    assert torch.equal(((words >> (a % 64)) & 1).bool(), legal)


def test_bounded_wait_gives_up_and_reports(ext):
    """The failure-detection path of the GEMM kernels' pipeline waits, on purpose: a
    wait on an mbarrier that nothing arrives on gives up after its limit (20 ms here),
    sets the error flag and returns; the context stays usable (a GEMM runs after)."""
    err, waited = ext.wait_timeout_probe(20_000_000)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert 20_000_000 <= int(waited.item()) < 1_000_000_000
    a = torch.randn((256, 512), device=DEV).to(torch.bfloat16)
    w = torch.randn((512, 512), device=DEV).to(torch.bfloat16)
    out = ext.linear(a, w, None)
    torch.cuda.synchronize()
    assert float((out.float() - a.float() @ w.float().t()).abs().max()) < 1.0
