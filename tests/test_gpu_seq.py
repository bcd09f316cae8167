"""GPU: the sequence policy's decode path (python/cugo_seq50.py, cugo_seq_attention50.py)
on the native kernels, against the reference's own outputs and fp32 restatements.

Tolerances.  decode attention writes bf16 (relative step 2^-8 of the value): it must
lie within 2^-8 |ref| + 1e-5 of the fp32 attention of the same bf16 inputs.
LayerNorm rounds to bf16 after fp32 math: within one bf16 step (2^-7 |ref|) + 1e-5.
Token embeddings are fp32 sums of bf16 weights: within 1e-5 relative + 1e-5.
The whole decoder (4 pre-LN layers, bf16 GEMM operands, bf16 KV cache) is checked
against the reference SeqNet's exact fp32 forward: its error must be no larger
(x1.5) than that of the reference's own forward under bf16 autocast, at most 2e-2
of the logit scale, and the argmax must agree wherever the top-2 margin exceeds 4x
that error.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from tests.seq_reference import attention_case, decode_attention_fp32, query_input

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _bf16(t):
    return t.to(DEV, torch.bfloat16)


def _close_bf16(out, ref, rel=2.0 ** -8, abs_=1e-5):
    diff = (out.float() - ref).abs()
    assert bool((diff <= rel * ref.abs() + abs_).all()), float(diff.max())


# ---- decode attention ------------------------------------------------------------

def test_decode_attention_matches_reference_golden(ext, golden):
    g = golden("seq_decode")
    q, k, v, pos, rows = attention_case(seed=3, n=48, n_rows=64)
    out = ext.decode_attention(_bf16(q), _bf16(k), _bf16(v), pos.to(DEV), rows.to(DEV))
    torch.cuda.synchronize()
    _close_bf16(out, torch.from_numpy(g["att_out"]).to(DEV))


@pytest.mark.parametrize("n,n_rows,slots,with_rows", [
    (1, 1, 1, False),          # a single slot
    (4096, 4096, 50, False),   # the reference cache: 50 slots, row i per query
    (5000, 700, 64, True),     # repeated rows (read-only), slots a multiple of 32
    (333, 1000, 100, True),    # more than two slot chunks per lane
    (257, 300, 512, True),     # the capacity limit
])
def test_decode_attention_matches_fp32(ext, n, n_rows, slots, with_rows):
    q, k, v, pos, rows = attention_case(seed=n + slots, n=n, n_rows=n_rows, slots=slots)
    if not with_rows:
        rows = torch.arange(n)
    out = ext.decode_attention(_bf16(q), _bf16(k), _bf16(v), pos.to(DEV),
                               rows.to(DEV) if with_rows else None)
    ref = decode_attention_fp32(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), rows.to(DEV))
    torch.cuda.synchronize()
    _close_bf16(out, ref)


def test_decode_attention_empty_batch(ext):
    q = torch.zeros((0, 8, 32), dtype=torch.bfloat16, device=DEV)
    kv = torch.zeros((4, 8, 50, 32), dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros(0, dtype=torch.int64, device=DEV)
    assert ext.decode_attention(q, kv, kv, pos).shape == (0, 8, 32)


def test_decode_attention_append_equals_put_then_attend(ext):
    n, n_rows, slots = 3000, 3000, 50
    q, k, v, pos, rows = attention_case(seed=9, n=n, n_rows=n_rows, slots=slots)
    g = torch.Generator().manual_seed(10)
    k_new = torch.randn((n, 8, 32), generator=g).to(torch.bfloat16)
    v_new = torch.randn((n, 8, 32), generator=g).to(torch.bfloat16)
    kc, vc = _bf16(k), _bf16(v)
    qkv = torch.cat((_bf16(q).view(n, 256), k_new.to(DEV).view(n, 256), v_new.to(DEV).view(n, 256)), 1)
    qd = qkv[:, :256].view(n, 8, 32)
    kd = qkv[:, 256:512].view(n, 8, 32)
    vd = qkv[:, 512:].view(n, 8, 32)
    out = ext.decode_attention(qd, kc, vc, pos.to(DEV), rows.to(DEV), k_new=kd, v_new=vd)
    # reference order: index_put_ the new key/value, then attend (python/cugo_seq50.py:313-317)
    k_ref, v_ref = _bf16(k).clone(), _bf16(v).clone()
    r_dev, p_dev = rows.to(DEV), pos.to(DEV)
    k_ref[r_dev, :, p_dev] = k_new.to(DEV)
    v_ref[r_dev, :, p_dev] = v_new.to(DEV)
    ref = decode_attention_fp32(q.to(DEV), k_ref.float(), v_ref.float(), p_dev, r_dev)
    torch.cuda.synchronize()
    assert torch.equal(kc, k_ref) and torch.equal(vc, v_ref)  # only slot pos of each row changed
    _close_bf16(out, ref)


def test_decode_attention_positions_from_lengths(ext):
    n_rows, slots = 2048, 50
    q, k, v, _, _ = attention_case(seed=12, n=1024, n_rows=n_rows, slots=slots)
    g = torch.Generator().manual_seed(13)
    length = torch.randint(0, 80, (n_rows,), generator=g)  # some past the clamp
    rows = torch.randperm(n_rows, generator=g)[:1024]
    clamp = 40
    out = ext.decode_attention(_bf16(q), _bf16(k), _bf16(v), length.to(DEV), rows.to(DEV),
                               pos_clamp=clamp)
    pos = length.index_select(0, rows).clamp_max(clamp)
    ref = decode_attention_fp32(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), rows.to(DEV))
    torch.cuda.synchronize()
    _close_bf16(out, ref)


def test_decode_attention_bad_position_reports_error(ext):
    q, k, v, pos, rows = attention_case(seed=14, n=64, n_rows=64, slots=50)
    pos[5] = 50      # past the last slot
    rows[7] = 64     # past the last row
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ext.decode_attention(_bf16(q), _bf16(k), _bf16(v), pos.to(DEV), rows.to(DEV), error=err)
    ref = decode_attention_fp32(q.to(DEV), k.to(DEV), v.to(DEV), pos.clamp_max(49).to(DEV),
                                rows.clamp_max(63).to(DEV))
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert not out[5].any() and not out[7].any()
    keep = torch.ones(64, dtype=torch.bool)
    keep[[5, 7]] = False
    _close_bf16(out[keep.to(DEV)], ref[keep.to(DEV)])


# ---- LayerNorm, GEMM modes, tokens -------------------------------------------------

@pytest.mark.parametrize("n,d", [(1, 256), (5000, 256), (777, 512), (64, 1024), (100, 128)])
def test_layernorm_matches_torch(ext, n, d):
    g = torch.Generator().manual_seed(n + d)
    x = (torch.randn((n, d), generator=g) * 3 + 1).to(DEV)
    w = (torch.rand(d, generator=g) + 0.5).to(DEV)
    b = (torch.randn(d, generator=g) * 0.1).to(DEV)
    out = ext.layernorm(x, w, b)
    ref = F.layer_norm(x, (d,), w, b, 1e-5)
    torch.cuda.synchronize()
    _close_bf16(out, ref, rel=2.0 ** -7)


@pytest.mark.parametrize("m,n,k", [(4096, 256, 256), (1000, 768, 256), (8192, 256, 1024)])
def test_linear_fp32_residual_stream_in_place(ext, m, n, k):
    g = torch.Generator().manual_seed(m)
    a = torch.randn((m, k), generator=g).to(DEV, torch.bfloat16)
    w = (torch.randn((n, k), generator=g) * k ** -0.5).to(DEV, torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(DEV)          # fp32 bias
    x = torch.randn((m, n), generator=g).to(DEV)                 # fp32 residual stream
    ref = x + a.float() @ w.float().t() + bias
    out = ext.linear(a, w, bias, residual=x, out=x)
    torch.cuda.synchronize()
    assert out.data_ptr() == x.data_ptr()
    diff = (x - ref).abs()
    assert bool((diff <= 1e-3 * ref.abs() + 1e-3).all()), float(diff.max())


def test_linear_gelu_epilogue(ext):
    g = torch.Generator().manual_seed(21)
    a = torch.randn((3000, 256), generator=g).to(DEV, torch.bfloat16)
    w = (torch.randn((1024, 256), generator=g) / 16).to(DEV, torch.bfloat16)
    bias = (torch.randn(1024, generator=g) * 0.1).to(DEV)
    out = ext.linear(a, w, bias, act=3)
    ref = F.gelu(a.float() @ w.float().t() + bias)
    torch.cuda.synchronize()
    diff = (out.float() - ref).abs()
    assert bool((diff <= 1e-2 * ref.abs() + 1e-2).all()), float(diff.max())


def _decoder(seed=11):
    from cugo_b200.seq import SeqDecoder
    return SeqDecoder.from_state_dict(SeqDecoder.random_state(seed=seed), device=DEV)


def test_tokens_match_reference_golden(golden):
    g = golden("seq_decode")
    dec = _decoder()
    start = torch.from_numpy(g["start"]).to(DEV)
    seat = torch.from_numpy(g["seat"]).to(DEV)
    events = torch.from_numpy(g["events"][:, 0].copy()).to(DEV)
    st = dec.start_token(start, seat)
    ev = dec.event_token(events, seat, torch.zeros_like(seat))
    torch.cuda.synchronize()
    for got, name in ((st, "start_tok"), (ev, "event_tok0")):
        ref = torch.from_numpy(g[name]).to(DEV)
        diff = (got - ref).abs()
        assert bool((diff <= 1e-5 * ref.abs() + 1e-5).all()), (name, float(diff.max()))


def test_observe_query_input(ext, golden):
    g = golden("steps")
    states = torch.from_numpy(g["rows"]).to(DEV)
    ids = torch.arange(states.size(0), device=DEV).flip(0)
    q, legal, player, done, status = ext.observe_query_bf16(states, ids)
    f32 = ext.observe_indexed(states, ids)
    torch.cuda.synchronize()
    assert torch.equal(q, query_input(f32[0], f32[1]))
    for a, b in zip((legal, player, done, status), f32[1:]):
        assert torch.equal(a, b)


# ---- the decoder against the reference SeqNet ---------------------------------------

def _inputs(g):
    keys = ("start", "seat", "events", "count", "features", "legal")
    t = {k: torch.from_numpy(np.ascontiguousarray(g[k])).to(DEV) for k in keys}
    t["max_count"] = int(g["count"].max())
    return t


def _run_decoder(dec, t):
    """The wave collector's incremental order on the golden positions (device inputs)."""
    b = t["count"].shape[0]
    cache = dec.new_cache(b)
    x = dec.start_token(t["start"], t["seat"])
    dec.cached_step(cache, x, slots=1)
    cache.length.fill_(1)
    for e in range(t["max_count"]):
        x = dec.event_token(t["events"][:, e].contiguous(), t["seat"],
                            torch.full((b,), e, dtype=torch.int64, device=DEV))
        dec.cached_step(cache, x)
        cache.length += (e < t["count"]).long()
    x = dec.query_token(query_input(t["features"], t["legal"]))
    dec.cached_step(cache, x, rows=torch.arange(b, device=DEV))
    return dec.readout(x)


def test_decoder_matches_reference_seqnet(golden):
    g = golden("seq_decode")
    logits = _run_decoder(_decoder(), _inputs(g))
    torch.cuda.synchronize()
    full = torch.from_numpy(g["logits_full"]).to(DEV)
    auto = torch.from_numpy(g["logits_autocast"]).to(DEV)
    err = (logits - full).abs().max().item()
    err_ref = (auto - full).abs().max().item()
    scale = full.abs().max().item()
    assert err <= 1.5 * err_ref + 1e-4, (err, err_ref)
    assert err <= 2e-2 * scale, (err, scale)
    top2 = full.topk(2, 1).values
    clear = (top2[:, 0] - top2[:, 1]) > 4 * err
    assert torch.equal(logits.argmax(1)[clear], full.argmax(1)[clear])


def test_events_query_decoder_matches_reference_seqnet(golden):
    """SeqNet in "events" mode (the query reads the context columns and the legal
    actions only): the same bar as the hybrid decoder against the reference's own
    fp32 forward (golden made by importing the reference's SeqNet)."""
    from cugo_b200.seq import SeqDecoder
    g = golden("seq_decode")
    dec = SeqDecoder.from_state_dict(SeqDecoder.random_state(seed=11, mode="events"), device=DEV)
    assert dec.mode == "events"
    logits = _run_decoder(dec, _inputs(g))
    torch.cuda.synchronize()
    full = torch.from_numpy(g["logits_events_full"]).to(DEV)
    auto = torch.from_numpy(g["logits_events_autocast"]).to(DEV)
    err = (logits - full).abs().max().item()
    err_ref = (auto - full).abs().max().item()
    assert err <= 1.5 * err_ref + 1e-4, (err, err_ref)
    assert err <= 2e-2 * full.abs().max().item()


def test_decoder_cuda_graph_replay_matches_eager(golden):
    t = _inputs(golden("seq_decode"))
    dec = _decoder()
    eager = _run_decoder(dec, t).clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _run_decoder(dec, t)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = _run_decoder(dec, t)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


# ---- the wave self-play driver --------------------------------------------------------

def _wave(graphs, wave=512):
    from cugo_b200.seq_selfplay import SeqWaveSelfPlay
    return SeqWaveSelfPlay(_decoder(seed=0), wave=wave, graphs=graphs)


def test_wave_selfplay_graph_replay_equals_eager(ext):
    runs = []
    for graphs in (False, True):
        sp = _wave(graphs)
        steps = sp.play_wave(game0=1000)
        torch.cuda.synchronize()
        runs.append((steps, sp.final_reward0.clone(), sp.count.clone(), sp.events.clone(),
                     sp.records["actions"].clone(), sp.finished.clone()))
        sp.release()
    (s0, *a), (s1, *b) = runs
    assert s0 == s1
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    assert bool(runs[0][5].all())


def _replay_wave(ext, sp, game0):
    """Replays a wave's recorded actions on fresh deals with step_events_indexed:
    (count, events, final reward, decisions, valid-as-expected) per game."""
    w = sp.w
    games = game0 + torch.arange(w, device=DEV)
    states = ext.create(12345 + games, games & 1)
    events = torch.zeros_like(sp.events)
    count = torch.zeros(w, dtype=torch.int64, device=DEV)
    reward = torch.zeros(w, device=DEV)
    decisions = torch.zeros(w, dtype=torch.int32, device=DEV)
    ids = torch.arange(w, device=DEV)
    acts = sp.records["actions"]
    expect_valid = torch.zeros_like(sp.records["valid"])
    learner_seat = (ids >> 1) & 1
    for s in range(acts.shape[0]):
        _, _, players, done, _ = ext.observe_indexed(states, ids)
        rows = ids[~done]
        if rows.numel() == 0:
            break
        mover = players[rows].long()
        mine = (rows >= sp.pool) | (mover == learner_seat[rows])
        expect_valid[s, rows] = mine
        r0, fin, _, status, committed, ev = ext.step_events_indexed(states, rows, acts[s, rows])
        assert bool((status == 0).all())
        c = rows[committed]
        events[c, count[c]] = ev[committed]
        count[c] += 1
        decisions[rows] += 1
        reward[rows[fin]] = r0[fin]
    assert bool(ext.observe(states)[3].all())
    return count, events, reward, decisions, expect_valid


@pytest.mark.parametrize("pool", [0, 128])
def test_wave_selfplay_records_replay_on_the_engine(ext, pool):
    """The wave-tail kernel's bookkeeping (event log, counts, final rewards, decision
    counters, records) against a replay of the recorded actions; with pool games the
    opponent decoder moves for its seat and only the learner's decisions are valid."""
    from cugo_b200.seq_selfplay import SeqWaveSelfPlay
    opponent = _decoder(seed=5) if pool else None
    sp = SeqWaveSelfPlay(_decoder(seed=0), wave=512, graphs=True, opponent=opponent,
                         pool_games=pool)
    sp.play_wave(game0=77)
    torch.cuda.synchronize()
    count, events, reward, decisions, expect_valid = _replay_wave(ext, sp, 77)
    assert torch.equal(count, sp.count)
    assert torch.equal(events, sp.events)
    assert torch.equal(reward, sp.final_reward0)
    assert torch.equal(decisions, sp.decision)
    assert torch.equal(expect_valid, sp.records["valid"])
    assert torch.equal(sp.cache.length, torch.cat((count, count)) + 1)
    if pool:
        assert int(sp.records["valid"][:, :pool].sum()) < int(decisions[:pool].sum())
    sp.release()


def _two_pass_driver(decoder, opponent, pool):
    """The wave step as two passes of the cached transformer per step -- the query
    tokens before the engine step, the event's tokens after it, the opening tokens in
    the reset -- the order the reference's WaveCollector runs them in."""
    from cugo_b200.seq_selfplay import SeqWaveSelfPlay

    class TwoPass(SeqWaveSelfPlay):
        def _reset(self):
            super()._reset()
            dec = self.dec
            self.cache.length.zero_()
            dec.cached_step(self.cache, self.x[:2 * self.w].clone(), slots=1)
            self.cache.length.fill_(1)
            if self.pool:
                self.opp_cache.length.zero_()
                self.opponent.cached_step(self.opp_cache, self.opp_x[:self.pool].clone(), slots=1)
                self.opp_cache.length.fill_(1)

        def _step(self):
            ext, dec, w, ids, st = self.ext, self.dec, self.w, self.ids, self.state
            query, legal, players, done, status = ext.observe_query_bf16(self.states, ids,
                                                                          query=self.query)
            seat = players.long() & 1
            x = dec.query_token(query)
            dec.cached_step(self.cache, x, rows=seat * w + ids)
            logits = dec.readout(x)
            if self.pool:
                p, opp = self.pool, self.opponent
                xo = opp.query_token(query[:p])
                opp.cached_step(self.opp_cache, xo)
                theirs = seat[:p] != self.learner_seat
                logits[:p] = torch.where(theirs.unsqueeze(1), opp.readout(xo)[:, :logits.shape[1]],
                                         logits[:p])
                self.learner[:p] = ~theirs
            actions, logp = ext.sample_actions(logits, legal, self.game0 + ids, st["decision"],
                                               seed_base=self.seed_base)
            self.rec_query.index_copy_(0, st["step_index"].clamp_max(self.max_steps - 1),
                                       query.unsqueeze(0))
            step_out = ext.step_events_indexed(self.states, ids, actions)
            events = step_out[5]
            dec.cached_step(self.cache, dec.event_token(events, self.seats2, st["count"]))
            if self.pool:
                p, opp = self.pool, self.opponent
                opp.cached_step(self.opp_cache,
                                opp.event_token(events[:p], self.opp_seat, st["count"][:p]))
                self.opp_cache.length += (step_out[4][:p] & ~done[:p]).long()
            ext.wave_tail(done, status, players, actions, logp, step_out, st, self.records,
                          learner=self.learner if self.pool else None)

    return TwoPass(decoder, wave=512, graphs=False, opponent=opponent, pool_games=pool)


@pytest.mark.parametrize("pool", [0, 128])
def test_wave_one_pass_equals_two_passes(ext, pool):
    """The driver runs the previous step's event tokens and this step's query tokens
    as one pass (shared LayerNorm and GEMM launches, the events' attention first at
    every layer); the same wave played with two passes per step records the same
    actions, log p and event logs."""
    from cugo_b200.seq_selfplay import SeqWaveSelfPlay
    runs = []
    for two in (False, True):
        opponent = _decoder(seed=5) if pool else None
        dec = _decoder(seed=0)
        sp = (_two_pass_driver(dec, opponent, pool) if two else
              SeqWaveSelfPlay(dec, wave=512, graphs=False, opponent=opponent, pool_games=pool))
        steps = sp.play_wave(game0=321)
        torch.cuda.synchronize()
        runs.append((steps, sp.records["actions"].clone(), sp.records["logp"].clone(),
                     sp.events.clone(), sp.final_reward0.clone()))
    (s0, *a), (s1, *b) = runs
    assert s0 == s1
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("slots", [50, 100])  # the staged kernel, then the warp-per-head one
def test_decode_attention_active_mask(ext, slots):
    """decode_attention restricted to active queries: those attend and append exactly as
    without the mask; the others get zeros, leave their cache rows untouched and set
    no error."""
    g = torch.Generator(device="cpu").manual_seed(3)
    n, rows_n, heads, dh = 2048, 4096, 8, 32
    kc = torch.randn((rows_n, heads, slots, dh), generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn((rows_n, heads, slots, dh), generator=g).to(DEV, torch.bfloat16)
    qkv = torch.randn((n, 3 * heads * dh), generator=g).to(DEV, torch.bfloat16)
    q, kn, vn = (qkv[:, i * 256:(i + 1) * 256].view(n, heads, dh) for i in range(3))
    length = torch.randint(0, slots, (rows_n,), generator=g).to(DEV)
    rows = torch.randperm(rows_n, generator=g)[:n].to(DEV)
    active = (torch.rand(n, generator=g) < 0.7).to(DEV)
    k0, v0 = kc.clone(), vc.clone()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = ext.decode_attention(q, k0, v0, length, rows=rows, k_new=kn, v_new=vn,
                               pos_clamp=slots - 1, error=err)
    for _ in range(2):  # the same result twice
        k1, v1 = kc.clone(), vc.clone()
        out = ext.decode_attention(q, k1, v1, length, rows=rows, k_new=kn, v_new=vn,
                                   pos_clamp=slots - 1, error=err, active=active)
        torch.cuda.synchronize()
        assert int(err) == 0
        assert torch.equal(out[active], ref[active])
        assert not bool(out[~active].float().abs().any())
        on, off = rows[active], rows[~active]
        assert torch.equal(k1[on], k0[on]) and torch.equal(v1[on], v0[on])
        assert torch.equal(k1[off], kc[off]) and torch.equal(v1[off], vc[off])


def test_decode_attention_invalid_rows_leave_the_others_alone(ext):
    """Queries with an out-of-range cache row take no ring space; the valid queries of
    the same launch get exactly what they get without them (an item without bytes must
    not misplace the ring's live data), and the error flag is set."""
    g = torch.Generator(device="cpu").manual_seed(8)
    n, rows_n, heads, slots, dh = 4096, 8192, 8, 50, 32
    kc = torch.randn((rows_n, heads, slots, dh), generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn((rows_n, heads, slots, dh), generator=g).to(DEV, torch.bfloat16)
    q = torch.randn((n, heads, dh), generator=g).to(DEV, torch.bfloat16)
    length = torch.randint(0, slots, (rows_n,), generator=g).to(DEV)
    rows = torch.randperm(rows_n, generator=g)[:n].to(DEV)
    bad = torch.rand(n, generator=g).to(DEV) < 0.3
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = ext.decode_attention(q, kc, vc, length, rows=rows, pos_clamp=slots - 1, error=err)
    torch.cuda.synchronize()
    assert int(err) == 0
    out = ext.decode_attention(q, kc, vc, length, rows=torch.where(bad, -1, rows),
                               pos_clamp=slots - 1, error=err)
    torch.cuda.synchronize()
    assert int(err) == 1
    assert torch.equal(out[~bad], ref[~bad])
    assert not bool(out[~bad].isnan().any()) and not bool(out[bad].float().abs().any())
