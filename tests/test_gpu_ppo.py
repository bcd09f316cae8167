"""GPU: the PPO update path (python/cugo_ppo50.py:514-745) on the fused GEMMs.

Gradients of FusedResidualMlp are compared with the same network in plain PyTorch:
their error against the exact fp32 gradients must be no larger (x1.5) than that of
the reference's own bf16-autocast backward, plus 1e-3 of the gradient scale.  A full
PPO minibatch step is compared with a restatement of the reference's step under
autocast: the three losses within 1e-2 relative and, per network, the clipped
gradients at cosine similarity >= 0.999.
"""
from __future__ import annotations

import pytest
import torch

from tests.torch_reference import TorchResidualMlp, ppo_losses_reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _twins(inputs, outputs, hidden=512, blocks=3, activation="silu", seed=0, squeeze=False):
    from cugo_b200.ppo import FusedResidualMlp
    torch.manual_seed(seed)
    ref = TorchResidualMlp(inputs, outputs, hidden, blocks, activation).to(DEV)
    with torch.no_grad():
        for p in ref.parameters():  # non-zero everywhere so every gradient flows
            p.copy_((torch.randn_like(p) * (1.0 / p.shape[-1]) ** 0.5).to(torch.bfloat16).float())
    fused = FusedResidualMlp(inputs, outputs, hidden, blocks, activation, squeeze=squeeze).to(DEV)
    fused.load_state_dict(ref.state_dict())  # same parameter names as the reference module
    return fused, ref


def _grads(module):
    return [p.grad.detach().float().clone() for p in module.parameters()]


@pytest.mark.parametrize("inputs,outputs,activation", [(720, 179, "silu"), (770, 1, "silu"),
                                                      (720, 179, "relu")])
def test_fused_mlp_gradients_match_torch(inputs, outputs, activation):
    fused, ref = _twins(inputs, outputs, activation=activation)
    g = torch.Generator().manual_seed(1)
    x = torch.randn((4096, inputs), generator=g).to(DEV, torch.bfloat16)
    r = torch.randn((4096, outputs), generator=g).to(DEV)
    (fused(x).float() * r).sum().backward()
    ours = _grads(fused)
    (ref(x.float()) * r).sum().backward()
    exact = _grads(ref)
    ref.zero_grad()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = ref(x.float())
    (out.float() * r).sum().backward()
    auto = _grads(ref)
    for (name, _), a, e, h in zip(fused.named_parameters(), ours, exact, auto):
        scale = float(e.abs().max())
        err, err_ref = float((a - e).abs().max()), float((h - e).abs().max())
        assert err <= 1.5 * err_ref + 1e-3 * scale, (name, err, err_ref, scale)


@pytest.mark.parametrize("inputs,outputs,activation", [(720, 179, "relu"), (770, 1, "silu"),
                                                      (770, 51, "silu")])
def test_inference_forward_matches_torch(inputs, outputs, activation):
    """Without autograd the activations run in the GEMM epilogues and a scalar head is a
    row reduction: the error against the fp32 module stays within that of the
    reference's bf16 autocast forward (x1.5 + 1e-3 of the output scale), and a
    second call (cached weights) is identical."""
    fused, ref = _twins(inputs, outputs, activation=activation, squeeze=outputs == 1)
    g = torch.Generator().manual_seed(5)
    x = torch.randn((3000, inputs), generator=g).to(DEV, torch.bfloat16)
    with torch.no_grad():
        ours = fused(x).float().reshape(3000, outputs)
        again = fused(x).float().reshape(3000, outputs)
        exact = ref(x.float())
        with torch.autocast("cuda", dtype=torch.bfloat16):
            auto = ref(x.float()).float()
    assert torch.equal(ours, again)
    scale = float(exact.abs().max())
    err, err_ref = float((ours - exact).abs().max()), float((auto - exact).abs().max())
    assert err <= 1.5 * err_ref + 1e-3 * scale, (err, err_ref, scale)
    with torch.no_grad():  # an in-place update of a weight is seen by the next call
        fused.out.weight.mul_(2.0)
        fused.out.bias.zero_()
        ref.out.weight.mul_(2.0)
        ref.out.bias.zero_()
        moved = fused(x).float().reshape(3000, outputs)
        exact2 = ref(x.float())
    assert float((moved - exact2).abs().max()) <= 2 * err + 2e-3 * float(exact2.abs().max())


def test_rowdot_matches_fp32():
    from cugo_b200 import load_extension
    ext = load_extension()
    g = torch.Generator().manual_seed(6)
    for m, k, ld in ((1, 8, 8), (37, 512, 520), (5000, 2048, 2048), (4099, 776, 776)):
        a = torch.randn((m, ld), generator=g).to(DEV, torch.bfloat16)
        w = torch.randn(k, generator=g).to(DEV)
        b = torch.randn(1, generator=g).to(DEV)
        out = ext.rowdot(a[:, :k], w, b)
        expect = a[:, :k].double() @ w.double() + b.double()
        assert torch.allclose(out.double(), expect, rtol=1e-5, atol=1e-4 * k ** 0.5)


def test_critic_input_and_squeeze():
    from cugo_b200.ppo import critic_input, fused_critic
    feats = torch.rand((5, 720), device=DEV).to(torch.bfloat16)
    hand = torch.tensor([0, 1, 3, (1 << 49), (1 << 50) - 1], device=DEV)
    x = critic_input(feats, hand)
    assert x.shape == (5, 770)
    assert torch.equal(x[:, :720], feats)
    for i, h in enumerate(hand.tolist()):
        assert x[i, 720:].tolist() == [float((h >> b) & 1) for b in range(50)]
    assert fused_critic().to(DEV)(x).shape == (5,)


def test_ppo_step_matches_reference_step():
    from cugo_b200.ppo import Minibatch, PpoStep, critic_input
    actor, actor_ref = _twins(720, 179, seed=2)
    critic, critic_ref = _twins(770, 1, seed=3, squeeze=True)
    g = torch.Generator().manual_seed(4)
    b = 8192
    legal = torch.rand((b, 179), generator=g) < 0.1
    legal[:, 0] = True
    logits0 = torch.randn((b, 179), generator=g)
    actions = torch.multinomial(torch.softmax(logits0.masked_fill(~legal, -1e30), 1), 1).squeeze(1)
    mb = Minibatch(features=torch.rand((b, 720), generator=g).to(DEV, torch.bfloat16),
                   legal=legal.to(DEV), actions=actions.to(DEV),
                   logp_old=(torch.randn(b, generator=g) * 0.1 - 2.0).to(DEV),
                   opp_hand=torch.randint(0, 1 << 50, (b,), generator=g).to(DEV),
                   adv=torch.randn(b, generator=g).to(DEV), ret=torch.randn(b, generator=g).to(DEV))
    opt = torch.optim.Adam(list(actor.parameters()) + list(critic.parameters()), lr=3e-4)
    step = PpoStep(actor, critic, opt)
    step.entropy_coef.fill_(0.05)
    ours = step.losses(mb)
    # reference step under autocast (python/cugo_ppo50.py:566-603)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = actor_ref(mb.features.float()).float()
        value = critic_ref(critic_input(mb.features, mb.opp_hand).float()).float().squeeze(-1)
    pl, vl, ent = ppo_losses_reference(logits, value, mb.legal, mb.actions, mb.logp_old, mb.adv, mb.ret, 0.2)
    for a, r in zip(ours[:3], (pl, vl, ent)):
        assert abs(float(a) - float(r)) <= 1e-2 * abs(float(r)) + 1e-4, (float(a), float(r))
    loss_ref = pl - 0.05 * ent + 0.5 * vl
    loss_ref.backward()
    step.step(mb)  # backward + clip + Adam on the fused networks
    for fused, ref in ((actor, actor_ref), (critic, critic_ref)):
        torch.nn.utils.clip_grad_norm_(list(ref.parameters()), 1.0)
        a = torch.cat([p.grad.flatten() for p in fused.parameters()])
        r = torch.cat([p.grad.flatten() for p in ref.parameters()])
        cos = float(torch.dot(a, r) / (a.norm() * r.norm()))
        assert cos >= 0.999, cos
    assert int(step.sums[5]) == 1


def test_graphed_step_equals_eager_step():
    from cugo_b200.ppo import GraphedPpoStep, Minibatch, PpoStep
    nets = []
    for _ in range(2):
        actor, _ = _twins(720, 179, seed=5)
        critic, _ = _twins(770, 1, seed=6, squeeze=True)
        opt = torch.optim.Adam(list(actor.parameters()) + list(critic.parameters()), lr=3e-4,
                               capturable=True)
        nets.append((actor, critic, PpoStep(actor, critic, opt)))
    g = torch.Generator().manual_seed(7)
    b = 4096

    def batch():
        legal = torch.rand((b, 179), generator=g) < 0.2
        legal[:, 0] = True
        return Minibatch(features=torch.rand((b, 720), generator=g).to(DEV, torch.bfloat16),
                         legal=legal.to(DEV), actions=torch.zeros(b, dtype=torch.int64, device=DEV),
                         logp_old=torch.full((b,), -1.5, device=DEV),
                         opp_hand=torch.randint(0, 1 << 50, (b,), generator=g).to(DEV),
                         adv=torch.randn(b, generator=g).to(DEV), ret=torch.randn(b, generator=g).to(DEV))

    batches = [batch() for _ in range(3)]
    graphed = GraphedPpoStep(nets[1][2], batches[0])
    for mb in batches:
        nets[0][2].step(mb)
        graphed(mb)
    torch.cuda.synchronize()
    for a, b2 in zip(list(nets[0][0].parameters()) + list(nets[0][1].parameters()),
                     list(nets[1][0].parameters()) + list(nets[1][1].parameters())):
        assert torch.allclose(a, b2, rtol=1e-5, atol=1e-6)
    assert torch.allclose(nets[0][2].sums, nets[1][2].sums, rtol=1e-5, atol=1e-6)


def _minibatch(b, seed):
    from cugo_b200.ppo import Minibatch
    g = torch.Generator().manual_seed(seed)
    legal = torch.rand((b, 179), generator=g) < 0.1
    legal[:, 0] = True
    logits0 = torch.randn((b, 179), generator=g)
    actions = torch.multinomial(torch.softmax(logits0.masked_fill(~legal, -1e30), 1), 1).squeeze(1)
    return Minibatch(features=torch.rand((b, 720), generator=g).to(DEV, torch.bfloat16),
                     legal=legal.to(DEV), actions=actions.to(DEV),
                     logp_old=(torch.randn(b, generator=g) * 0.1 - 2.0).to(DEV),
                     opp_hand=torch.randint(0, 1 << 50, (b,), generator=g).to(DEV),
                     adv=torch.randn(b, generator=g).to(DEV), ret=torch.randn(b, generator=g).to(DEV))


@pytest.mark.parametrize("activation", ["silu", "relu"])
def test_native_step_gradients_match_reference(activation):
    """The native step (train_forward, the fused loss kernel, train_backward) against
    the reference's step restated in PyTorch under bf16 autocast: the three losses
    and the KL / clip-fraction statistics within 1e-2 relative, every parameter's
    gradient (before clipping) within 1.5x the autocast gradient's own error against
    fp32 plus 1e-3 of its scale, and per network cosine >= 0.999."""
    from cugo_b200.ppo import NativePpoStep, critic_input, train_backward, train_forward
    actor, actor_ref = _twins(720, 179, seed=2, activation=activation)
    critic, critic_ref = _twins(770, 1, seed=3, squeeze=True, activation=activation)
    mb = _minibatch(8192, 4)
    opt = torch.optim.Adam(list(actor.parameters()) + list(critic.parameters()), lr=3e-4)
    step = NativePpoStep(actor, critic, opt)
    step.entropy_coef.fill_(0.05)
    ext = actor.ext
    logits, a_saved = train_forward(actor, mb.features)
    value, c_saved = train_forward(critic, critic_input(mb.features, mb.opp_hand))
    dy = torch.empty((8192, 184), dtype=torch.bfloat16, device=DEV)
    dv = torch.empty(8192, device=DEV)
    stats = torch.zeros(5, device=DEV)
    ext.ppo_loss(logits, mb.legal, mb.actions, mb.logp_old, mb.adv, value, mb.ret, 0.2,
                 step.entropy_coef, 0.5, dy, dv, stats)
    train_backward(actor, a_saved, dy=dy)
    train_backward(critic, c_saved, dv=dv)
    assert not dy[:, 179:].any()

    def reference(autocast: bool):
        for net in (actor_ref, critic_ref):
            net.zero_grad()
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            lg = actor_ref(mb.features.float()).float()
            v = critic_ref(critic_input(mb.features, mb.opp_hand).float()).float().squeeze(-1)
        pl, vl, ent = ppo_losses_reference(lg, v, mb.legal, mb.actions, mb.logp_old, mb.adv, mb.ret, 0.2)
        (pl - 0.05 * ent + 0.5 * vl).backward()
        lp = torch.log_softmax(lg.masked_fill(~mb.legal, -1.0e30), 1).gather(
            1, mb.actions.unsqueeze(1)).squeeze(1)
        r = (lp - mb.logp_old).exp()
        kl = ((r - 1) - (lp - mb.logp_old)).mean()
        cf = ((r - 1).abs() > 0.2).float().mean()
        grads = [p.grad.detach().float().clone() for n in (actor_ref, critic_ref) for p in n.parameters()]
        return [float(x) for x in (pl, vl, ent, kl, cf)], grads

    stats_auto, g_auto = reference(True)
    _, g_exact = reference(False)
    for got, want in zip(stats.tolist(), stats_auto):
        assert abs(got - want) <= 1e-2 * abs(want) + 1e-4, (got, want)
    ours = [p.grad.detach().float() for n in (actor, critic) for p in n.parameters()]
    names = [f"actor.{n}" for n, _ in actor.named_parameters()] + \
            [f"critic.{n}" for n, _ in critic.named_parameters()]
    for name, a, h, e in zip(names, ours, g_auto, g_exact):
        scale = float(e.abs().max())
        err, err_ref = float((a - e).abs().max()), float((h - e).abs().max())
        assert err <= 1.5 * err_ref + 1e-3 * scale, (name, err, err_ref, scale)
    for k0, k1 in ((0, len(list(actor.parameters()))), (len(list(actor.parameters())), len(ours))):
        a = torch.cat([t.flatten() for t in ours[k0:k1]])
        r = torch.cat([t.flatten() for t in g_exact[k0:k1]])
        assert float(torch.dot(a, r) / (a.norm() * r.norm())) >= 0.999


def test_native_graphed_step_equals_eager_step():
    from cugo_b200.ppo import GraphedPpoStep, NativePpoStep
    nets = []
    for _ in range(2):
        actor, _ = _twins(720, 179, seed=5)
        critic, _ = _twins(770, 1, seed=6, squeeze=True)
        opt = torch.optim.Adam(list(actor.parameters()) + list(critic.parameters()), lr=3e-4,
                               capturable=True)
        nets.append((actor, critic, NativePpoStep(actor, critic, opt)))
    batches = [_minibatch(4096, 10 + i) for i in range(3)]
    graphed = GraphedPpoStep(nets[1][2], batches[0])
    for mb in batches:
        nets[0][2].step(mb)
        graphed(mb)
    torch.cuda.synchronize()
    for a, b2 in zip(list(nets[0][0].parameters()) + list(nets[0][1].parameters()),
                     list(nets[1][0].parameters()) + list(nets[1][1].parameters())):
        assert torch.allclose(a, b2, rtol=1e-5, atol=1e-6)
    assert torch.allclose(nets[0][2].sums, nets[1][2].sums, rtol=1e-4, atol=1e-6)
    assert int(nets[0][2].sums[5]) == 3
