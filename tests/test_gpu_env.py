"""GPU parity: the CUDA batch environment (through libcugo_b200.so's C ABI) against
the oracle and the committed golden fixtures."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests import differential as dif

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def t(a, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a))
    return x.to(device=DEV, dtype=dtype) if dtype else x.to(DEV)


def n(x):
    return x.cpu().numpy()


class GpuImpl:
    """numpy-in/numpy-out adapter of the extension ops (for tests.differential)."""

    def __init__(self, ext):
        self.ext = ext

    def create(self, seeds, first):
        return n(self.ext.create(t(seeds, torch.int64), t(first, torch.int64)))

    def observe(self, rows):
        out = self.ext.observe(t(rows))
        return tuple(n(x) for x in out)

    def step(self, rows, actions, events=False):
        states = t(rows)
        ids = torch.arange(states.size(0), device=DEV)
        out = self.ext.step_events_indexed(states, ids, t(actions, torch.int64))
        res = (n(states),) + tuple(n(x) for x in out[:5])
        return res + (n(out[5]),) if events else res

    def start(self, rows):
        return n(self.ext.start(t(rows)))

    def stock(self, rows):
        s = t(rows)
        return n(self.ext.stock_indexed(s, torch.arange(s.size(0), device=DEV)))


def test_constants(ext):
    assert (ext.FEATURE_COUNT, ext.ACTION_COUNT, ext.PRIMARY_ACTION_COUNT, ext.CHOICE_ACTION_BEGIN,
            ext.EVENT_WORDS, ext.START_WORDS, ext.STATE_BYTES, ext.STATUS_OK) == (
                720, 179, 127, 127, 9, 8, 248, 0)


def test_create_golden(ext, golden):
    c = golden("create")
    assert np.array_equal(n(ext.create(t(c["seeds"]), t(c["first"]))), c["rows"])


def test_observe_golden(ext, golden):
    g = golden("steps")
    f, legal, player, done, status = (n(x) for x in ext.observe(t(g["rows"])))
    assert np.abs(f - g["features"]).max() <= 1e-6
    assert np.array_equal(legal, g["legal"])
    assert np.array_equal(player, g["player"]) and np.array_equal(done, g["done"])
    assert np.array_equal(status, g["status"])
    # observe_indexed through a permutation reproduces the same rows.
    perm = np.random.default_rng(0).permutation(g["rows"].shape[0])
    fi, li, pi, di, si = (n(x) for x in ext.observe_indexed(t(g["rows"]), t(perm)))
    assert np.array_equal(fi, f[perm]) and np.array_equal(li, legal[perm])
    assert np.array_equal(pi, player[perm]) and np.array_equal(si, status[perm])


def test_step_golden(ext, golden):
    g = golden("steps")
    states = t(g["rows"])
    reward, done, nagari, status, committed = (n(x) for x in ext.step(states, t(g["actions"])))
    assert np.array_equal(n(states), g["next_rows"])
    assert np.array_equal(reward, g["reward"]) and np.array_equal(done, g["step_done"])
    assert np.array_equal(nagari, g["nagari"]) and np.array_equal(status, g["step_status"])
    assert np.array_equal(committed, g["committed"])
    states = t(g["rows"])
    ids = torch.arange(states.size(0), device=DEV)
    out = ext.step_events_indexed(states, ids, t(g["actions"]))
    assert np.array_equal(n(out[5]), g["events"])
    assert np.array_equal(n(states), g["next_rows"])


def test_reads_golden(ext, golden):
    g = golden("steps")
    s = t(g["rows"])
    ids = torch.arange(s.size(0), device=DEV)
    assert np.array_equal(n(ext.start(s)), g["start"])
    assert np.array_equal(n(ext.stock_indexed(s, ids)), g["stock"])
    assert np.array_equal(n(ext.hands_indexed(s, ids)), g["hands"])


def test_config0_rollouts_golden(ext, golden):
    """Config 0 on the GPU: games 0..4095 played to the end by the seeded
    random-legal rule give the oracle's event hashes and results."""
    g = golden("config0")
    r = {k: n(v) for k, v in ext.rollout_random(0, 4096, seed_base=12345, max_decisions=256).items()}
    assert np.array_equal(r["hashes"].view(np.uint64), g["hashes"])
    assert np.array_equal(r["reward0"], g["reward0"])
    assert np.array_equal(r["decisions"], g["decisions"])
    assert np.array_equal(r["events"], g["events"])
    assert np.array_equal(r["last_status"], g["last_status"])
    assert np.array_equal(r["final_rows"][:256], g["final_rows_head"])


@pytest.mark.parametrize("family,salt", [(0, 1), (1, 2), (2, 3)])
def test_random_play_matches_oracle(ext, oracle, family, salt):
    stats = dif.play_against_oracle(GpuImpl(ext), oracle, n=8192, family=family, salt=salt)
    assert stats["done"] > 0.99


def test_rollouts_match_oracle_at_scale(ext, oracle):
    r = {k: n(v) for k, v in ext.rollout_random(100_000, 65536, seed_base=12345).items()}
    o = oracle.rollout_random(100_000, 65536, seed_base=12345)
    for key in ("reward0", "decisions", "events", "last_status", "final_rows"):
        assert np.array_equal(r[key], o[key]), key
    assert np.array_equal(r["hashes"].view(np.uint64), o["hashes"])


def test_branch_roots_golden(ext, golden):
    g = golden("roots")
    roots = ext.branch_roots(256, seed_base=12345)
    assert np.array_equal(n(roots), g["roots"])
    ids, actions = ext.branch_actions(roots, 4, seed_base=12345)
    assert np.array_equal(n(ids), g["ids"]) and np.array_equal(n(actions), g["actions"])


def test_branch_children_match_oracle(ext, oracle):
    """Config 2 at reduced size: every child equals the oracle's clone + step."""
    roots = ext.branch_roots(2048, seed_base=12345)
    ids, actions = ext.branch_actions(roots, 16, seed_base=12345)
    child, reward, done, nagari, status, committed = (n(x) for x in ext.branch_indexed(roots, ids, actions))
    parents = n(roots)[n(ids)]
    o = oracle.step(parents, n(actions))
    assert np.array_equal(child, o[0])
    for a, b in zip((reward, done, nagari, status, committed), o[1:]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("ragged", [0, 100, 300])
def test_branch_config2_windows_match_oracle(ext, oracle, ragged):
    """Config 2's layout (256 branches per root, one root per warp's group of
    entries): every child and output equals the oracle's clone + step, including a
    ragged end inside a group and inside a block's last warp."""
    roots = ext.branch_roots(301, seed_base=4242)
    ids, actions = ext.branch_actions(roots, 256, seed_base=4242)
    m = ids.numel() - ragged
    ids, actions = ids[:m].contiguous(), actions[:m].contiguous()
    out = [n(x) for x in ext.branch_indexed(roots, ids, actions)]
    o = oracle.step(n(roots)[n(ids)], n(actions))
    assert np.array_equal(out[0], o[0])
    for a, b in zip(out[1:], o[1:]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("layout", ["all_actions", "shuffled", "repeats"])
def test_branch_entries_of_every_layout_match_oracle(ext, oracle, layout):
    """branch_indexed makes each distinct (parent, action) child once per 256 entries
    and copies it to the others: every entry equals the oracle's clone + step whether
    the entries are all distinct (every legal action of consecutive rows: two passes
    of a block), shuffled, or heavy repeats, with invalid ids and actions mixed in and
    a ragged last block."""
    roots = ext.branch_roots(1500, seed_base=777)
    legal = n(ext.observe(roots)[1])
    rows, acts = np.nonzero(legal)
    rng = np.random.default_rng(5)
    if layout == "shuffled":
        perm = rng.permutation(rows.size)
        rows, acts = rows[perm], acts[perm]
    elif layout == "repeats":
        pick = rng.integers(0, rows.size, size=20000)
        pick.sort()
        rows, acts = rows[pick], acts[pick]
    rows, acts = rows.astype(np.int64), acts.astype(np.int64)
    bad = rng.random(rows.size) < 0.01
    rows[bad] = rng.choice([-1, 1500, 10**9], size=int(bad.sum()))
    bad_act = rng.random(rows.size) < 0.01
    acts[bad_act] = rng.choice([-1, 179, 1000], size=int(bad_act.sum()))
    m = rows.size - 37  # a ragged last block
    rows, acts = rows[:m], acts[:m]
    out = [n(x) for x in ext.branch_indexed(roots, torch.from_numpy(rows).to(DEV),
                                            torch.from_numpy(acts).to(DEV))]
    valid = (rows >= 0) & (rows < 1500)
    parents = np.zeros((m, 248), dtype=np.uint8)
    parents[valid] = n(roots)[rows[valid]]
    o = oracle.step(parents, acts)
    assert np.array_equal(out[0][valid], o[0][valid])
    assert not out[0][~valid].any()
    for a, b in zip(out[1:], o[1:]):
        assert np.array_equal(a[valid], b[valid])
    assert (out[4][~valid] == -1).all() and out[2][~valid].all()


def test_selfplay_step_matches_oracle(ext, oracle):
    """Config 1 at reduced size: slots 0..4095 of generation 0 follow the oracle's
    games; the features written are observe()'s."""
    slots = 4096
    seeds = torch.arange(slots, device=DEV, dtype=torch.int64) + 12345
    states = ext.create(seeds, torch.arange(slots, device=DEV) & 1)
    slot_game = torch.arange(slots, device=DEV, dtype=torch.int64)
    slot_decision = torch.zeros(slots, dtype=torch.int32, device=DEV)
    completed = torch.zeros(slots, dtype=torch.int32, device=DEV)
    steps = torch.zeros(slots, dtype=torch.int64, device=DEV)
    features = torch.empty((slots, 720), dtype=torch.float32, device=DEV)
    legal = torch.empty((slots, 179), dtype=torch.bool, device=DEV)
    k = 8
    for i in range(k):
        before = states.clone()
        ext.selfplay_random_step(states, slot_game, slot_decision, completed, steps, features, legal)
    f, l, _, _, _ = ext.observe(before)
    # The last launch observed `before` unless a slot was reset in that launch.
    same = n(slot_game) == np.arange(slots)
    assert np.abs(n(features)[same] - n(f)[same]).max() <= 1e-6
    assert np.array_equal(n(legal)[same], n(l)[same])
    o = oracle.rollout_random(0, slots, seed_base=12345, max_decisions=k)
    live = same & (o["decisions"] == k)
    assert live.mean() > 0.9
    assert np.array_equal(n(states)[live], o["final_rows"][live])
    assert np.array_equal(n(slot_decision)[live], o["decisions"][live])


def test_branch_semantics(ext):
    """The reference's branch conformance checks (python/branch50_smoke.py:101-164)."""
    seeds = torch.arange(4096, device=DEV, dtype=torch.int64) * 7919 + 3
    parents = ext.create(seeds, torch.arange(4096, device=DEV) & 1)
    f, legal, _, done, status = ext.observe(parents)
    keep = torch.nonzero((~done) & (status == 0)).flatten()
    parents = parents.index_select(0, keep).contiguous()
    legal = legal.index_select(0, keep)
    ext.step(parents, legal.to(torch.int64).argmax(1))
    _, legal, _, done, status = ext.observe(parents)
    keep = torch.nonzero((~done) & (status == 0)).flatten()
    parents = parents.index_select(0, keep).contiguous()
    count = parents.size(0)
    snapshot = parents.clone()
    clone_ids = torch.tensor([0, 7, 0, 3, 7, 1], device=DEV)
    assert torch.equal(ext.clone_indexed(parents, clone_ids), parents.index_select(0, clone_ids))
    assert torch.equal(parents, snapshot)

    def clone_step(ids, acts):
        children = ext.clone_indexed(parents, ids)
        return [children] + list(ext.step(children, acts))

    ids = torch.arange(1024, device=DEV).mul(37).remainder(count)
    _, bl, _, bd, bs = ext.observe_indexed(parents, ids)
    assert not bool(bd.any()) and not bool((bs != 0).any())
    acts = bl.to(torch.int64).argmax(1)
    for a, b in zip(ext.branch_indexed(parents, ids, acts), clone_step(ids, acts)):
        assert torch.equal(a, b)
    assert torch.equal(parents, snapshot)
    # invalid parent ids: zero children and the invalid-id step outputs
    bad = torch.tensor([-1, count], device=DEV)
    zeros = torch.zeros(2, dtype=torch.int64, device=DEV)
    out = ext.branch_indexed(parents, bad, zeros)
    ref_states = parents.clone()
    exp = ext.step_indexed(ref_states, bad, zeros)
    for a, b in zip(out[1:], exp):
        assert torch.equal(a, b)
    assert not bool(out[0].any())
    assert torch.equal(ref_states, parents)
    assert n(exp[3]).tolist() == [-1, -1] and n(exp[1]).tolist() == [True, True]
    # invalid actions
    two = torch.tensor([0, 1], device=DEV)
    bad_actions = torch.tensor([-1, 179], device=DEV)
    for a, b in zip(ext.branch_indexed(parents, two, bad_actions), clone_step(two, bad_actions)):
        assert torch.equal(a, b)
    assert torch.equal(parents, snapshot)


def test_empty_batches(ext):
    s = ext.create(torch.tensor([5], device=DEV), torch.tensor([0], device=DEV))
    e = torch.empty(0, dtype=torch.int64, device=DEV)
    assert tuple(ext.clone_indexed(s, e).shape) == (0, 248)
    out = ext.branch_indexed(s, e, e)
    assert tuple(out[0].shape) == (0, 248) and all(x.numel() == 0 for x in out[1:])
    assert ext.observe_indexed(s, e)[0].shape == (0, 720)
    assert all(x.numel() == 0 for x in ext.step_indexed(s, e, e))
    empty_states = ext.create(e, e)
    assert tuple(empty_states.shape) == (0, 248)
    assert ext.observe(empty_states)[1].shape == (0, 179)
    assert ext.start(empty_states).shape == (0, 8)


def test_invalid_index_observation(ext):
    s = ext.create(torch.tensor([5, 6], device=DEV), torch.tensor([0, 1], device=DEV))
    f, legal, player, done, status = ext.observe_indexed(s, torch.tensor([-1, 2, 1], device=DEV))
    assert not bool(f[:2].any()) and not bool(legal[:2].any())
    assert n(player[:2]).tolist() == [0, 0] and n(done[:2]).tolist() == [True, True]
    assert n(status[:2]).tolist() == [-1, -1]
    assert int(status[2]) == 0
    h = ext.hands_indexed(s, torch.tensor([-1, 0], device=DEV))
    assert n(h[0]).tolist() == [0, 0] and int(h[1, 0]) != 0
    assert int(ext.stock_indexed(s, torch.tensor([9], device=DEV))[0]) == -1


def test_ops_capture_in_cuda_graph(ext):
    seeds = torch.arange(2048, device=DEV, dtype=torch.int64)
    states = ext.create(seeds, seeds & 1)
    eager = states.clone()
    ids = torch.arange(2048, device=DEV)
    _, legal, _, _, _ = ext.observe(states)
    acts = legal.to(torch.int64).argmax(1)
    eager_out = ext.step_indexed(eager, ids, acts)
    f_eager = ext.observe(eager)[0]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ext.observe(states)  # warm the allocator on this stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ext.step_indexed(states, ids, acts)
        feat = ext.observe(states)[0]
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(states, eager)
    assert torch.equal(feat, f_eager)
    for a, b in zip(out, eager_out):
        assert torch.equal(a, b)


# Byte ranges of a finished row that record how the game went (the TorchEnv50 image:
# end reason at 129, shaken months 104..107, bombs 108, bomb credits 110, ppuk count
# 120, go count 96, Gukjin role 102, nagari 240).
RARE_FIELDS = {"shaken": (104, 4), "bombs": (108, 2), "credits": (110, 2), "ppuk": (120, 2),
               "go": (96, 2)}


def test_rare_rule_paths_at_scale(ext, oracle):
    """A million seeded random-legal games (games 0 .. 2^20 - 1), every final row,
    reward, decision count and event hash bit-exact with the reference's engine.
    The range holds every way a game ends — Stop, Chongtong at the deal, on the
    floor and by a bonus replacement, three ppuk, nagari — each at least 100 times,
    and games with shakes, bombs, bomb credits, ppuk and Go calls."""
    games = 1 << 20
    r = {k: n(v) for k, v in ext.rollout_random(0, games, seed_base=12345).items()}
    o = oracle.rollout_random(0, games, seed_base=12345)
    for key in ("reward0", "decisions", "events", "last_status", "final_rows"):
        assert np.array_equal(r[key], o[key]), key
    assert np.array_equal(r["hashes"].view(np.uint64), o["hashes"])
    rows = r["final_rows"]
    reasons = np.bincount(rows[:, 129], minlength=6)
    # 1 Stop, 2 dealt Chongtong, 3 floor Chongtong, 4 bonus-replacement Chongtong, 5 three ppuk
    assert all(reasons[k] >= 100 for k in (1, 2, 3, 4, 5)), reasons
    assert int(rows[:, 240].sum()) >= 100  # nagari
    for name, (off, width) in RARE_FIELDS.items():
        assert int(np.any(rows[:, off:off + width] != 0, axis=1).sum()) >= 100, name
