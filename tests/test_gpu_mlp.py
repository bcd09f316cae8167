"""GPU: the tcgen05 GEMM layer and the residual-MLP policy against fp32 references.

Tolerances.  Outputs are bf16-rounded (relative step 2^-8) and hidden states are
bf16 between layers, as under the reference's bf16 autocast.  A single layer is
checked to 1% relative + 1e-2 absolute of the fp32 product of the same bf16
operands.  The whole policy is checked against the exact fp32 forward: its error
must be no larger (x1.25) than that of the reference's own forward under bf16
autocast (python/cugo_ppo50.py:366) and at most 1% of the logit scale, every
decision whose best action leads by more than 4x that error must pick the same
action, and overall argmax agreement must be at least the reference's own.  (A
fixed 99.9% agreement between two bf16 computations is not attainable on random
weights: the reference's autocast forward itself agrees with the exact forward on
only ~99.6% of decisions because of near ties.)
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from tests.torch_reference import mlp_forward_autocast, mlp_forward_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _rand(shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(DEV, torch.bfloat16)


@pytest.mark.parametrize("m,n,k,act,act_after,res,fp32", [
    (1000, 512, 720, 0, 0, False, False),     # input layer, ragged M and K
    (4096, 512, 512, 1, 0, False, False),     # fc1 + ReLU
    (4097, 512, 512, 0, 0, True, False),      # fc2 + residual
    (3000, 512, 512, 0, 2, True, False),      # last block: residual then SiLU
    (777, 180, 512, 0, 0, False, True),       # head, fp32 out, ragged N
    (128, 64, 720, 2, 0, False, False),       # narrow layer
    (300_000, 512, 512, 1, 0, False, False),  # many persistent tiles per SM
    (4096, 256, 256, 0, 0, False, False),     # 64-column tiles (32 wide ones for 148 SMs)
    (8192, 256, 256, 2, 0, False, False),     # 128-column tiles
    (4096, 256, 1024, 0, 0, True, True),      # long K, fp32 residual: 64-column tiles, not pairs
    (1000, 200, 256, 1, 0, True, False),      # narrow tiles with ragged N and a residual
])
def test_linear_matches_fp32(ext, m, n, k, act, act_after, res, fp32):
    a = _rand((m, k), 1.0, 1)
    w = _rand((n, k), (2.0 / k) ** 0.5, 2)
    b = _rand((n,), 0.1, 3)
    r = _rand((m, n), 1.0, 4) if res else None
    if res and fp32:  # the residual has the output's dtype
        r = r.float()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ext.linear(a, w, b, residual=r.clone() if res else None, act=act, act_after=act_after,
                     out_dtype=torch.float32 if fp32 else torch.bfloat16, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    acts = {0: lambda x: x, 1: F.relu, 2: F.silu}
    ref = acts[act](a.float() @ w.float().t() + b.float())
    if res:
        ref = ref + r.float()
    ref = acts[act_after](ref)
    diff = (out.float() - ref).abs()
    assert bool((diff <= 1e-2 * ref.abs() + 1e-2).all()), float(diff.max())


def test_linear_in_place_residual(ext):
    a = _rand((2048, 512), 1.0, 5)
    w = _rand((512, 512), 0.06, 6)
    h = _rand((2048, 512), 1.0, 7)
    expect = (a.float() @ w.float().t()) + h.float()
    ext.linear(a, w, None, residual=h, out=h)
    assert float((h.float() - expect).abs().max()) <= 0.05


def _observations(ext, rows=65536):
    """Distinct mid-game observations from the config-1 driver."""
    idx = torch.arange(rows, device=DEV, dtype=torch.int64)
    states = ext.create(idx + 777, idx & 1)
    game, dec = idx.clone(), torch.zeros(rows, dtype=torch.int32, device=DEV)
    done_n, steps = torch.zeros_like(dec), torch.zeros(rows, dtype=torch.int64, device=DEV)
    feats = torch.empty((rows, 720), dtype=torch.float32, device=DEV)
    legal = torch.empty((rows, 179), dtype=torch.bool, device=DEV)
    for _ in range(6):
        ext.selfplay_random_step(states, game, dec, done_n, steps, feats, legal)
    return feats, legal


@pytest.mark.parametrize("hidden,blocks,act", [(512, 3, "relu"), (512, 3, "silu"), (2048, 4, "relu")])
def test_policy_matches_reference_forward(ext, hidden, blocks, act):
    from cugo_b200.policy import ResidualMlpPolicy

    pol = ResidualMlpPolicy(hidden, blocks, act, device=DEV, seed=0)
    # Non-zero biases exercise the fused bias path.
    pol.biases = [_rand(b.shape, 0.05, 10 + i) for i, b in enumerate(pol.biases)]
    feats, legal = _observations(ext)
    out = pol(feats)
    exact = mlp_forward_fp32(pol.weights, pol.biases, feats, blocks, act)
    auto = mlp_forward_autocast(pol.weights, pol.biases, feats, blocks, act)
    scale = max(1.0, float(exact.abs().max()))
    err = (out - exact).abs()
    err_ref = (auto - exact).abs()
    assert float(err.max()) <= 1.25 * float(err_ref.max()) + 1e-3
    assert float(err.mean()) <= 1.25 * float(err_ref.mean()) + 1e-4
    assert float(err.max()) <= 1e-2 * scale
    live = legal.any(1)

    def greedy(x):
        return x[:, :179].masked_fill(~legal, -1e30).argmax(1)

    top2 = exact[:, :179].masked_fill(~legal, -1e30).topk(2, dim=1).values
    one_legal = legal.sum(1) == 1
    clear = live & (one_legal | ((top2[:, 0] - top2[:, 1]) > 4 * float(err.max())))
    assert bool((greedy(out) == greedy(exact))[clear].all())
    agree = float((greedy(out) == greedy(exact))[live].float().mean())
    agree_ref = float((greedy(auto) == greedy(exact))[live].float().mean())
    assert agree >= agree_ref - 1e-3, (agree, agree_ref)


def test_reference_ppo_actor_golden(golden):
    """Logits of the reference's own PpoActor (hidden 64, 2 blocks, SiLU) loaded
    through from_state_dict."""
    from cugo_b200.policy import ResidualMlpPolicy

    gd = golden("ppo_actor_64x2")
    state = {k: torch.from_numpy(v).view(torch.bfloat16) for k, v in gd.items() if k != "logits"}
    pol = ResidualMlpPolicy.from_state_dict(state, blocks=2, activation="silu", device=DEV)
    feats = torch.from_numpy(golden("steps")["features"]).to(DEV)
    out = pol(feats).cpu()
    ref = torch.from_numpy(gd["logits"])
    scale = max(1.0, float(ref.abs().max()))
    assert float((out - ref).abs().max()) <= 2e-2 * scale


def test_policy_logit_bar_at_the_reference_init(ext, capsys):
    """The north_star bar on the 65,536 real observation rows: max |delta logit| <= 2e-2
    against the exact fp32 forward, with the networks at the reference's own
    initialisation scale (PpoActor's nn.Linear default init: uniform in +-1/sqrt(fan
    in), every layer non-zero, SiLU, 3 blocks of 512; bf16 weights), and argmax
    agreement reported beside the reference's autocast forward.  The agreement is
    asserted against the autocast forward's own (>= it - 0.1%); on random weights
    near ties bound any bf16 implementation below a fixed 99.9% (see the module
    docstring).  The measured figures are printed."""
    from cugo_b200.policy import ResidualMlpPolicy

    pol = ResidualMlpPolicy(512, 3, "silu", device=DEV, seed=0)
    g = torch.Generator().manual_seed(0)
    for i, (w, b) in enumerate(zip(pol.weights, pol.biases)):
        bound = 1.0 / w.shape[1] ** 0.5
        pol.weights[i] = ((torch.rand(w.shape, generator=g) * 2 - 1) * bound).to(DEV, torch.bfloat16)
        pol.biases[i] = ((torch.rand(b.shape, generator=g) * 2 - 1) * bound).to(DEV, torch.bfloat16)
    feats, legal = _observations(ext)
    out = pol(feats)[:, :179]
    exact = mlp_forward_fp32(pol.weights, pol.biases, feats, 3, "silu")[:, :179]
    auto = mlp_forward_autocast(pol.weights, pol.biases, feats, 3, "silu")[:, :179]
    live = legal.any(1)

    def greedy(x):
        return x.masked_fill(~legal, -1e30).argmax(1)

    err = float((out - exact).abs().max())
    err_auto = float((auto - exact).abs().max())
    agree = float((greedy(out) == greedy(exact))[live].float().mean())
    agree_auto = float((greedy(auto) == greedy(exact))[live].float().mean())
    agree_pair = float((greedy(out) == greedy(auto))[live].float().mean())
    with capsys.disabled():
        print(f"\nlogit bar (65,536 rows, {int(live.sum())} with a legal action): "
              f"max|dlogit| vs fp32 {err:.5f} (autocast {err_auto:.5f}, logit scale "
              f"{float(exact.abs().max()):.3f}); argmax agreement vs fp32 {agree:.5f} "
              f"(autocast {agree_auto:.5f}); vs autocast {agree_pair:.5f}")
    assert err <= 2e-2
    assert agree >= agree_auto - 1e-3


@pytest.mark.parametrize("m,n,k,act", [(32768, 512, 512, 2), (1000, 512, 720, 1), (300, 2048, 2048, 2)])
def test_linear_pre_keeps_the_pre_activation(ext, m, n, k, act):
    """linear_pre writes act(a w^T + b) and a w^T + b from one GEMM launch: each
    equals the plain layer's output (no activation / with it) bit for bit."""
    a = _rand((m, k), seed=1).to(DEV, torch.bfloat16)
    w = _rand((n, k), scale=k ** -0.5, seed=2).to(DEV, torch.bfloat16)
    b = _rand((n,), seed=3).to(DEV)
    pre = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    out = ext.linear_pre(a, w, b, act, pre)
    assert torch.equal(pre, ext.linear(a, w, b))
    assert torch.equal(out, ext.linear(a, w, b, act=act))
