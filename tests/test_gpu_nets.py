"""GPU: the network variants train_ppo50.py exposes, against the reference's own
modules (python/cugo_ppo_nets50.py, staged unmodified in baseline/_ref/python):
LayerNorm trunks (--norm layer), the belief head (--belief-coef) and value-bin critics
(--value-bins, the two-hot target).  As for the norm "none" networks, our error
against the exact fp32 result must be no larger (x1.5) than that of the reference's
own bf16-autocast run, plus a small fraction of the scale."""
from __future__ import annotations

import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def nets():
    from baseline import build_ref
    if not build_ref.available():
        pytest.fail("reference modules are not staged (python -m baseline.build_ref)")
    path = str(build_ref.reference_python())
    if path not in sys.path:
        sys.path.insert(0, path)
    import cugo_ppo_nets50
    return cugo_ppo_nets50


def _randomize(module: torch.nn.Module, seed: int) -> torch.nn.Module:
    """Every parameter non-zero and bf16-representable, so every gradient flows and
    both sides start from the same weights."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            if name.endswith("norm.weight") or ".0.weight" in name:
                v = 1.0 + 0.2 * torch.randn(p.shape, generator=g)
            else:
                v = torch.randn(p.shape, generator=g) * (1.0 / p.shape[-1]) ** 0.5
            p.copy_(v.to(torch.bfloat16).float())
    return module.to(DEV)


def _grads(module):
    return [p.grad.detach().float().clone() for p in module.parameters()]


def _check_against(ours_fn, ref_module, ref_fn, x, r, named, tol=1.5):
    """Forward outputs and gradients of `ours_fn` within tol x the reference autocast
    error of the exact fp32 values (plus 1e-3 of the scale)."""
    out = ours_fn()
    (out.float() * r).sum().backward()
    exact_out = ref_fn(x.float())
    (exact_out.float() * r).sum().backward()
    exact = _grads(ref_module)
    ref_module.zero_grad()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        auto_out = ref_fn(x.float())
    (auto_out.float() * r).sum().backward()
    auto = _grads(ref_module)
    scale = float(exact_out.detach().abs().max())
    err = float((out.float() - exact_out.detach()).abs().max())
    err_ref = float((auto_out.float() - exact_out.detach()).abs().max())
    assert err <= tol * err_ref + 1e-3 * scale, ("output", err, err_ref, scale)
    for (name, p), e, h in zip(named, exact, auto):
        a = p.grad.detach().float()
        gs = float(e.abs().max())
        err, err_ref = float((a - e).abs().max()), float((h - e).abs().max())
        assert err <= tol * err_ref + 1e-3 * gs, (name, err, err_ref, gs)


@pytest.mark.parametrize("kind", ["actor", "critic"])
def test_layernorm_network_matches_reference(nets, kind):
    from cugo_b200.ppo import critic_input, fused_actor, fused_critic
    if kind == "actor":
        ref = _randomize(nets.PpoActor(512, 3, "layer"), seed=1)
        ours = fused_actor(norm="layer").to(DEV)
    else:
        ref = _randomize(nets.OracleCritic(512, 3, "layer"), seed=2)
        ours = fused_critic(norm="layer").to(DEV)
    ours.load_state_dict(ref.state_dict())  # the reference's parameter names
    g = torch.Generator().manual_seed(3)
    m = 4096
    feats = torch.rand((m, 720), generator=g).to(DEV, torch.bfloat16)
    x = feats if kind == "actor" else critic_input(feats, torch.randint(0, 1 << 50, (m,), generator=g).to(DEV))
    outputs = 179 if kind == "actor" else 1
    r = torch.randn((m, outputs) if outputs > 1 else (m,), generator=g).to(DEV)
    # Inference (fp32 residual stream, the native row LayerNorm) against fp32 and autocast.
    with torch.no_grad():
        inf = ours(x).float()
        exact = ref(x.float()).float()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            auto = ref(x.float()).float()
    scale = float(exact.abs().max())
    err, err_ref = float((inf - exact).abs().max()), float((auto - exact).abs().max())
    assert err <= 1.5 * err_ref + 1e-3 * scale, ("inference", err, err_ref, scale)
    # Training forward and gradients, layer by layer on the tcgen05 kernels.
    _check_against(lambda: ours(x), ref, ref, x, r, list(ours.named_parameters()))


def test_belief_head_matches_reference(nets):
    from cugo_b200.ppo import FusedBeliefHead
    ref = _randomize(nets.BeliefHead(512, 512), seed=5)
    ours = FusedBeliefHead(512, 512).to(DEV)
    ours.load_state_dict(ref.state_dict())
    g = torch.Generator().manual_seed(6)
    h = (torch.randn((4096, 512), generator=g) * 2.0).to(DEV, torch.bfloat16).requires_grad_(True)
    r = torch.randn((4096, 50), generator=g).to(DEV)
    out = ours(h)
    (out * r).sum().backward()
    dh = h.grad.float().clone()
    h.grad = None
    hf = h.detach().float().requires_grad_(True)
    exact = ref(hf)
    (exact * r).sum().backward()
    dh_exact = hf.grad.clone()
    exact_grads = _grads(ref)
    ref.zero_grad()
    ha = h.detach().float().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        auto = ref(ha)
    (auto.float() * r).sum().backward()
    auto_grads = _grads(ref)
    for a, e, hh, name in ((out.float(), exact, auto.float(), "logits"), (dh, dh_exact, ha.grad, "dh")):
        s = float(e.abs().max())
        err, err_ref = float((a - e.detach()).abs().max()), float((hh - e.detach()).abs().max())
        assert err <= 1.5 * err_ref + 1e-3 * s, (name, err, err_ref, s)
    for (name, p), e, hh in zip(ours.named_parameters(), exact_grads, auto_grads):
        a = p.grad.float()
        s = float(e.abs().max())
        err, err_ref = float((a - e).abs().max()), float((hh - e).abs().max())
        assert err <= 1.5 * err_ref + 1e-3 * s, (name, err, err_ref, s)


def test_two_hot_and_card_plane_match_reference(nets):
    from cugo_b200.ppo import card_plane, fused_critic, two_hot
    critic = fused_critic(value_bins=51).to(DEV)
    support = critic.support
    assert torch.equal(support.cpu(), nets.value_support(51, 640.0))
    g = torch.Generator().manual_seed(7)
    y = (torch.randn(10000, generator=g) * 200.0).to(DEV)
    y[:3] = torch.tensor([-1e4, 1e4, 0.0], device=DEV)  # clamped at both ends
    ours, ref = two_hot(y, support), nets.two_hot(y, support)
    assert float((ours - ref).abs().max()) <= 1e-6
    assert float(((ours * support).sum(1) - y.clamp(float(support[0]), float(support[-1]))).abs().max()) <= 1e-3
    hands = torch.randint(0, 1 << 50, (1000,), generator=g).to(DEV)
    assert torch.equal(card_plane(hands), nets.card_plane(hands, torch.float32))


def test_step_with_belief_and_value_bins(nets):
    """A PpoStep with a LayerNorm actor, a belief head and a value-bin critic: its
    losses equal the reference composition's (python/cugo_ppo50.py:558-611) under
    autocast on the same weights within 1e-2, every network (the belief head
    included) receives gradients, and the belief loss is recorded."""
    from cugo_b200.ppo import FusedBeliefHead, Minibatch, PpoStep, critic_input, fused_actor, fused_critic
    actor_ref = _randomize(nets.PpoActor(512, 3, "layer"), seed=11)
    critic_ref = _randomize(nets.OracleCritic(512, 3, "none", value_bins=51), seed=12)
    belief_ref = _randomize(nets.BeliefHead(512, 512), seed=13)
    actor, critic, belief = fused_actor(norm="layer").to(DEV), fused_critic(value_bins=51).to(DEV), \
        FusedBeliefHead(512, 512).to(DEV)
    for a, b in ((actor, actor_ref), (critic, critic_ref), (belief, belief_ref)):
        a.load_state_dict(b.state_dict())
    g = torch.Generator().manual_seed(14)
    n = 4096
    legal = torch.rand((n, 179), generator=g) < 0.1
    legal[:, 0] = True
    mb = Minibatch(features=torch.rand((n, 720), generator=g).to(DEV, torch.bfloat16),
                   legal=legal.to(DEV), actions=torch.zeros(n, dtype=torch.int64, device=DEV),
                   logp_old=torch.full((n,), -2.0, device=DEV),
                   opp_hand=torch.randint(0, 1 << 50, (n,), generator=g).to(DEV),
                   adv=torch.randn(n, generator=g).to(DEV), ret=(torch.randn(n, generator=g) * 30).to(DEV))
    params = [*actor.parameters(), *critic.parameters(), *belief.parameters()]
    step = PpoStep(actor, critic, torch.optim.Adam(params, lr=3e-4), belief=belief, belief_coef=0.5)
    pl, vl, ent, _, _, bl = step.losses(mb)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits, hidden = actor_ref.forward_hidden(mb.features.float())
        belief_logits = belief_ref(hidden).float()
        value = critic_ref(critic_input(mb.features, mb.opp_hand).float()).float()
    logits = logits.float()
    lp = torch.log_softmax(logits.masked_fill(~mb.legal, -1.0e30), 1)
    ratio = (lp.gather(1, mb.actions.unsqueeze(1)).squeeze(1) - mb.logp_old).exp()
    pl_ref = -torch.min(ratio * mb.adv, ratio.clamp(0.8, 1.2) * mb.adv).mean()
    ent_ref = -(lp.exp() * lp).sum(1).mean()
    vl_ref = -(nets.two_hot(mb.ret, critic_ref.support) * torch.log_softmax(value, -1)).sum(-1).mean()
    bl_ref = torch.nn.functional.binary_cross_entropy_with_logits(
        belief_logits, nets.card_plane(mb.opp_hand, torch.float32))
    for a, r in ((pl, pl_ref), (vl, vl_ref), (ent, ent_ref), (bl, bl_ref)):
        assert abs(float(a) - float(r)) <= 1e-2 * abs(float(r)) + 1e-4, (float(a), float(r))
    step.step(mb)
    for net in (actor, critic, belief):
        assert all(p.grad is not None and bool(p.grad.abs().sum() > 0) for p in net.parameters())
    assert float(step.sums[6]) > 0 and int(step.sums[5]) == 1
