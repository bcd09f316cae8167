"""GPU: the reference's own callers, unmodified, on this extension.

The reference's python/ modules are staged unmodified in baseline/_ref/python, and its
own extension (python/csrc/torch50_ext.cpp/.cu) is built for sm_100 into
baseline/_ref/torch50_ext, by baseline/build_ref.py.  Every reference caller obtains
its extension from cugo_torch50_ext.load_extension(); the tests patch that loader to
return cugo_b200.load_extension() — the one-line swap a user makes — and run each
caller as written:

  torch50_smoke.main, branch50_smoke.main     the reference's own self-checking scripts
  cugo_ppo50.collect                          plain, with a pool opponent, with critic Q
                                              (action_values, OracleCritic with stock
                                              planes) and with redealt-world Q
                                              (redeal_worlds editing raw row words,
                                              _greedy_to_end, _child_values)
  cugo_eval50.evaluate_paired                 greedy and sampled
  cugo_seq_selfplay50.WaveCollector.collect   wave 512 with pool games

Where the caller's result is data, the same call with the same torch seed on the
reference's own extension is the expected value, and every output must be identical:
the engine ops are bit-exact, so the networks see the same inputs and the samplers
draw the same actions.
"""
from __future__ import annotations

import sys
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def ref():
    from baseline import build_ref
    if not build_ref.available():
        pytest.fail("reference modules and extension are not staged (python -m baseline.build_ref)")
    path = str(build_ref.reference_python())
    if path not in sys.path:
        sys.path.insert(0, path)
    import branch50_smoke
    import cugo_eval50
    import cugo_ppo50
    import cugo_ppo_nets50
    import cugo_seq50
    import cugo_seq_selfplay50
    import cugo_torch50_ext
    import torch50_smoke
    import train_seq50
    return SimpleNamespace(ext=build_ref.load_reference_extension(), loader=cugo_torch50_ext,
                           ppo=cugo_ppo50, nets=cugo_ppo_nets50, eval=cugo_eval50,
                           seq=cugo_seq50, wave=cugo_seq_selfplay50, train_seq=train_seq50,
                           branch_smoke=branch50_smoke, torch_smoke=torch50_smoke)


@pytest.fixture()
def swapped(ref, ext, monkeypatch):
    """The reference loader returning this package's extension."""
    monkeypatch.setattr(ref.loader, "load_extension", lambda *a, **k: ext)
    for mod in (ref.branch_smoke, ref.torch_smoke):
        monkeypatch.setattr(mod, "load_extension", ref.loader.load_extension)
    return ref.loader.load_extension()


def _init(model: torch.nn.Module, seed: int) -> torch.nn.Module:
    """Non-zero weights (the reference zero-initialises residual branches and heads)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in model.parameters():
            fan_in = p.shape[-1] if p.dim() > 1 else 64
            p.copy_(torch.randn(p.shape, generator=g) * (1.0 / fan_in) ** 0.5)
    return model.to(DEV).eval()


def test_swap_is_the_cugo_extension(ref, swapped):
    from cugo_b200.ext import CugoB200Extension
    assert isinstance(swapped, CugoB200Extension)
    for name in ("FEATURE_COUNT", "ACTION_COUNT", "PRIMARY_ACTION_COUNT", "CHOICE_ACTION_BEGIN",
                 "EVENT_WORDS", "START_WORDS", "STATE_BYTES", "STATUS_OK"):
        assert int(getattr(swapped, name)) == int(getattr(ref.ext, name)), name


def test_torch50_smoke_runs_unchanged(ref, swapped, monkeypatch, capsys):
    monkeypatch.setattr(sys, "argv", ["torch50_smoke.py", "--batch", "16384", "--hidden", "256",
                                      "--warmup", "1", "--iters", "1"])
    ref.torch_smoke.main()
    out = capsys.readouterr().out
    assert "smoke PASS" in out and "benchmark PASS" in out


def test_branch50_smoke_runs_unchanged(ref, swapped, monkeypatch, capsys):
    monkeypatch.setattr(sys, "argv", ["branch50_smoke.py", "--parents", "4096", "--batch", "65536",
                                      "--warmup", "1", "--iters", "2"])
    ref.branch_smoke.main()
    out = capsys.readouterr().out
    assert "correctness PASS" in out and "benchmark PASS" in out


def _rollout_equal(a, b) -> None:
    for name in ("features", "legal", "actions", "logp", "opp_hand", "stock", "returns"):
        x, y = getattr(a, name), getattr(b, name)
        assert x.shape == y.shape, name
        assert torch.equal(x, y), name
    for name in ("games", "terminal", "nagari", "decision_steps"):
        assert getattr(a, name) == getattr(b, name), name
    for name in ("mean_abs_reward0", "learner_score"):
        x, y = getattr(a, name), getattr(b, name)
        assert x == y or (x != x and y != y), name


COLLECT_CASES = {
    "plain": dict(games=8192),
    "pool": dict(games=8192, pool=True, pool_fraction=0.5, pool_greedy=True),
    "critic_q": dict(games=2048, all_actions=True, q_source="critic", critic_stock=True,
                     branch_max_top=0.9),
    "worlds_greedy": dict(games=512, all_actions=True, q_source="worlds", worlds=2, world_depth=0,
                          pool=True, pool_fraction=0.5, branch_max_top=0.9, branch_fraction=0.25),
    "worlds_critic": dict(games=1024, all_actions=True, q_source="worlds", worlds=3, world_depth=1,
                          worlds_first=2, branch_max_top=0.9),
}


@pytest.mark.parametrize("case", sorted(COLLECT_CASES))
def test_collect_equals_the_reference_extension(ref, swapped, case):
    c = dict(COLLECT_CASES[case])
    games = c.pop("games")
    all_actions = c.pop("all_actions", False)
    pool = [_init(ref.nets.PpoActor(256, 2, norm="none"), 3)] if c.pop("pool", False) else []
    pool_fraction = c.pop("pool_fraction", 0.0)
    pool_greedy = c.pop("pool_greedy", False)
    stock = c.pop("critic_stock", False)
    critic = _init(ref.nets.OracleCritic(256, 2, norm="none", stock=stock), 4) if all_actions else None
    actor = _init(ref.nets.PpoActor(256, 2, norm="none"), 2)
    results = []
    for ext in (swapped, ref.ext):
        storage = ref.ppo.RolloutStorage(games * 24, DEV, all_actions=all_actions)
        torch.manual_seed(77)
        r = ref.ppo.collect(ext, actor, pool, games, 1234, pool_fraction, pool_greedy, 32.0,
                            storage, critic=critic, **c)
        extra = tuple(t[:storage.size].clone() for t in storage.extra)
        results.append((r, extra))
    (mine, mine_extra), (theirs, theirs_extra) = results
    _rollout_equal(mine, theirs)
    assert mine.decision_steps > 10
    for x, y in zip(mine_extra, theirs_extra):
        assert torch.equal(torch.nan_to_num(x, nan=-7.0), torch.nan_to_num(y, nan=-7.0))
    if all_actions:
        q = mine_extra[0]
        assert int((~torch.isnan(q)).sum()) > games  # actions were branched and valued


@pytest.mark.parametrize("sample", [False, True])
def test_evaluate_paired_equals_the_reference_extension(ref, swapped, sample):
    a = _init(ref.nets.PpoActor(256, 2, norm="none"), 5)
    b = _init(ref.nets.PpoActor(256, 2, norm="none"), 6)
    out = []
    for ext in (swapped, ref.ext):
        torch.manual_seed(5)
        out.append(ref.eval.evaluate_paired(ext, a, b, 4096, 4321, 128, True,
                                            sample_a=sample, sample_b=sample))
    mine, theirs = out
    fields = [f for f in vars(mine) if f != "seconds"]
    assert fields
    for f in fields:
        x, y = getattr(mine, f), getattr(theirs, f)
        assert x == y or (x != x and y != y), f
    assert mine.games == 8192


def test_wave_collector_equals_the_reference_extension(ref, swapped):
    """WaveCollector (python/cugo_seq_selfplay50.py:36-238), hybrid SeqNet, wave 512,
    128 pool games per wave, two waves; the Triton decode kernel runs inside its CUDA
    graph in both runs."""
    seq = ref.seq
    actor = _init(seq.seq_actor("hybrid", 256, 4, 8), 8)
    opponent = ref.wave.make_opponent_slot(actor, lambda: seq.seq_actor("hybrid", 256, 4, 8))
    opp_state = {k: v.clone() for k, v in _init(seq.seq_actor("hybrid", 256, 4, 8), 9).state_dict().items()}
    games, wave = 1024, 512
    runs = []
    for ext in (swapped, ref.ext):
        collector = ref.wave.WaveCollector(ext, actor, opponent, wave, 128, None)
        storage = ref.train_seq.SeqStorage(games * 32, DEV)
        log = ref.wave.GameLog(games, DEV)
        torch.manual_seed(21)
        out = collector.collect(games, 99, opp_state, storage, log)
        collector.graph = None
        runs.append((storage, log, out))
    (s0, l0, o0), (s1, l1, o1) = runs
    assert s0.size == s1.size > games
    for name in ref.train_seq.SeqStorage.NAMES:
        assert torch.equal(getattr(s0, name)[:s0.size], getattr(s1, name)[:s1.size]), name
    for name in ("events", "count", "start"):
        assert torch.equal(getattr(l0, name), getattr(l1, name)), name
    for key in o0:
        x, y = o0[key], o1[key]
        assert (torch.equal(x, y) if isinstance(x, torch.Tensor) else x == y), key
