"""Incremental inference of the event-sequence policy on the native kernels.

`SeqDecoder` runs the decode half of the reference's ``SeqNet``
(python/cugo_seq50.py:131-339), query mode "hybrid" or "events" (the events query reads
the context columns only: its first layer's weight is zero on the other features), with
opening, event and query tokens
and ``cached_step`` — one new token per cache row through the pre-LN transformer
layers with the token's key/value appended to the row's KV cache — and the
``readout`` head.  Per layer:

    a   = LayerNorm1(x)                       layernorm kernel        (fp32 -> bf16)
    qkv = a . W_in^T + b_in                   tcgen05 GEMM            (bf16 [n, 3d])
    att = attend(q; cache + appended k, v)    decode-attention kernel (bf16 [n, d])
    x  += att . W_out^T + b_out               tcgen05 GEMM, fp32 residual in place
    a   = LayerNorm2(x)
    f   = GELU(a . W_1^T + b_1)               tcgen05 GEMM, GELU epilogue
    x  += f . W_2^T + b_2                     tcgen05 GEMM, fp32 residual in place

Numerics follow the reference under bf16 autocast: GEMM operands bf16 with fp32
accumulation, LayerNorm and softmax in fp32, the residual stream x in fp32 (the
reference's x becomes fp32 when its fp32 position/type parameters are added),
the KV cache bf16.  Opening and event tokens are multi-hot vectors; they are
embedded by gather-sum kernels over the transposed input weights.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .ext import load_extension

MAX_EVENTS = 48  # python/cugo_seq50.py:34
FEATURES = 720
ACTIONS = 179
QUERY_IN = FEATURES + ACTIONS  # hybrid query input (python/cugo_seq50.py:152-153)
# Feature columns the "events" query reads (python/cugo_contract50.py:34-36, contract
# v4): the decision context of contract v3, then the own hand, the table counts and
# the round multiplier.  The column list is the feature contract checkpoints are
# trained on, so it is the reference's.
EVENTS_CONTEXT = [*range(200, 250), *range(396, 453), *range(471, 476), 552,
                  *range(0, 50), *range(491, 496), 557, 710, 711]
EVENTS_QUERY_IN = len(EVENTS_CONTEXT) + ACTIONS
QUERY_LD = 904                 # query rows padded to a multiple of 16 bytes
ACT_GELU = 3


def decode_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, pos: torch.Tensor,
                     use_triton: bool = True, rows: torch.Tensor | None = None) -> torch.Tensor:
    """Drop-in for the reference's decode_attention (python/cugo_seq_attention50.py:43-57):
    q [n, heads, 32]; keys/values [rows, heads, slots, 32] bf16 (contiguous); pos, rows
    int64 [n] (rows defaults to 0..n-1) -> [n, heads, 32] in q's dtype.  `use_triton` is
    accepted for signature compatibility; the native kernel always runs (q is read as
    bf16, as the reference's callers pass it under autocast)."""
    del use_triton
    out = load_extension().decode_attention(q.to(torch.bfloat16), keys, values, pos.contiguous(),
                                            None if rows is None else rows.contiguous())
    return out if q.dtype == torch.bfloat16 else out.to(q.dtype)


def encode_events(h, length: int, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """Drop-in for the reference's encode_events (python/cugo_seq50.py:91-109) on the
    device: h has .events int64 [B, MAX_EVENTS, 9], .count [B], .seat [B]; returns the
    observer-relative tokens [B, length, 414] (fp32 or bf16) and their validity mask."""
    ext = load_extension()
    return ext.encode_events(h.events.contiguous(), h.count.contiguous(), h.seat.contiguous(),
                             length, dtype)


@dataclass
class _Layer:
    norm1_w: torch.Tensor
    norm1_b: torch.Tensor
    w_in: torch.Tensor   # bf16 [3d, d]
    b_in: torch.Tensor   # fp32 [3d]
    w_out: torch.Tensor  # bf16 [d, d]
    b_out: torch.Tensor
    norm2_w: torch.Tensor
    norm2_b: torch.Tensor
    w1: torch.Tensor     # bf16 [ffn, d]
    b1: torch.Tensor
    w2: torch.Tensor     # bf16 [d, ffn]
    b2: torch.Tensor


class SeqKVCache:
    """Keys/values of every cached token per row and layer (python/cugo_seq50.py:325-339):
    k, v bf16 [layers, rows, heads, slots, dh]; length int64 [rows]."""

    def __init__(self, decoder: "SeqDecoder", rows: int, slots: int = MAX_EVENTS + 2) -> None:
        dev = decoder.device
        self.heads, self.slots = decoder.heads, slots
        shape = (decoder.layers, rows, decoder.heads, slots, decoder.d_model // decoder.heads)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros_like(self.k)
        self.length = torch.zeros(rows, dtype=torch.int64, device=dev)
        self.rows = rows


class SeqDecoder:
    """SeqNet's incremental API (start_token, event_token, query_token,
    cached_step, readout) on tcgen05 GEMMs and the decode kernels."""

    def __init__(self, params: dict[str, torch.Tensor], layers: int, heads: int,
                 device: torch.device | str = "cuda", eps: float = 1e-5) -> None:
        self.ext = load_extension()
        self.device = torch.device(device)
        dev = self.device
        f32 = dict(dtype=torch.float32, device=dev)

        def bf16(t: torch.Tensor) -> torch.Tensor:
            return t.detach().to(dev, torch.bfloat16).contiguous()

        def fp32(t: torch.Tensor) -> torch.Tensor:
            return t.detach().to(**f32).contiguous()

        p = params
        self.layers, self.heads, self.eps = layers, heads, eps
        self.d_model = p["position"].shape[1]
        d = self.d_model
        if d // heads != 32:
            raise ValueError("the decode kernel needs 32-wide heads")
        self.position = fp32(p["position"])        # [MAX_EVENTS + 1, d]
        self.token_type = fp32(p["token_type"])    # [3, d]
        self.event_wt = bf16(p["event_in.weight"].t())   # [414, d]
        self.event_b = fp32(p["event_in.bias"])
        self.start_wt = bf16(p["start_in.weight"].t())   # [274, d]
        self.start_b = fp32(p["start_in.bias"])
        q0 = p["query_in.0.weight"].detach().float().cpu()
        w = torch.zeros((q0.shape[0], QUERY_LD), dtype=torch.float32)
        if q0.shape[1] == QUERY_IN:  # "hybrid": every feature and the legal actions
            self.mode = "hybrid"
            w[:, :QUERY_IN] = q0
        elif q0.shape[1] == EVENTS_QUERY_IN:
            # "events": the context columns and the legal actions.  The query input
            # keeps the hybrid layout (observe_query_bf16 writes all 720 features);
            # the other feature columns get zero weights, so the layer is the
            # reference's product over the selected columns.
            self.mode = "events"
            ctx = len(EVENTS_CONTEXT)
            w[:, EVENTS_CONTEXT] = q0[:, :ctx]
            w[:, FEATURES:QUERY_IN] = q0[:, ctx:]
        else:
            raise ValueError("query_in.0 must read the hybrid (720 + 179) or events "
                             f"({len(EVENTS_CONTEXT)} + 179) query")
        self.q_w0 = bf16(w)
        self.q_b0 = fp32(p["query_in.0.bias"])
        self.q_w1 = bf16(p["query_in.2.weight"])
        # query_in(...) + token_type[2]: the type row folds into the fp32 bias.
        self.q_b1 = fp32(p["query_in.2.bias"].detach().float().cpu() + p["token_type"].detach().float().cpu()[2])
        self.blocks: list[_Layer] = []
        for i in range(layers):
            pre = f"encoder.layers.{i}."
            self.blocks.append(_Layer(
                fp32(p[pre + "norm1.weight"]), fp32(p[pre + "norm1.bias"]),
                bf16(p[pre + "self_attn.in_proj_weight"]), fp32(p[pre + "self_attn.in_proj_bias"]),
                bf16(p[pre + "self_attn.out_proj.weight"]), fp32(p[pre + "self_attn.out_proj.bias"]),
                fp32(p[pre + "norm2.weight"]), fp32(p[pre + "norm2.bias"]),
                bf16(p[pre + "linear1.weight"]), fp32(p[pre + "linear1.bias"]),
                bf16(p[pre + "linear2.weight"]), fp32(p[pre + "linear2.bias"])))
        self.norm_w, self.norm_b = fp32(p["norm.weight"]), fp32(p["norm.bias"])
        self.h_w0, self.h_b0 = bf16(p["head.0.weight"]), fp32(p["head.0.bias"])
        h2 = p["head.2.weight"]
        self.outputs = h2.shape[0]
        self.out_ld = (self.outputs + 3) // 4 * 4  # fp32 rows in 16-byte multiples
        self.h_w1, self.h_b1 = bf16(h2), fp32(p["head.2.bias"])

    # -- construction -------------------------------------------------------------
    @classmethod
    def from_state_dict(cls, state: dict[str, torch.Tensor], heads: int = 8,
                        device: torch.device | str = "cuda") -> "SeqDecoder":
        """Loads a reference SeqNet state dict, mode "hybrid" or "events" (weights
        rounded to bf16)."""
        layers = len({k.split(".")[2] for k in state if k.startswith("encoder.layers.")})
        return cls(state, layers, heads, device)

    @staticmethod
    def random_state(seed: int = 0, d_model: int = 256, layers: int = 4, ffn: int = 1024,
                     outputs: int = ACTIONS, mode: str = "hybrid") -> dict[str, torch.Tensor]:
        """A SeqNet-shaped state dict drawn from torch.manual_seed(seed): nn.Linear's
        default U(-1/sqrt(in), 1/sqrt(in)) weights and biases, N(0, 0.02) position and
        token-type tables, LayerNorm weight 1 and bias 0 (python/cugo_seq50.py:154-166)."""
        g = torch.Generator().manual_seed(seed)

        def lin(name: str, out_f: int, in_f: int) -> dict[str, torch.Tensor]:
            b = 1.0 / math.sqrt(in_f)
            return {name + ".weight": (torch.rand((out_f, in_f), generator=g) * 2 - 1) * b,
                    name + ".bias": (torch.rand((out_f,), generator=g) * 2 - 1) * b}

        d = d_model
        st: dict[str, torch.Tensor] = {}
        st.update(lin("event_in", d, 8 * 50 + 12 + 2))
        st.update(lin("start_in", d, 5 * 50 + 12 + 8 + 4))
        st.update(lin("query_in.0", 2 * d, QUERY_IN if mode == "hybrid" else EVENTS_QUERY_IN))
        st.update(lin("query_in.2", d, 2 * d))
        st["position"] = torch.randn((MAX_EVENTS + 1, d), generator=g) * 0.02
        st["token_type"] = torch.randn((3, d), generator=g) * 0.02
        for i in range(layers):
            pre = f"encoder.layers.{i}."
            inp = lin(pre + "self_attn.in_proj", 3 * d, d)
            st[pre + "self_attn.in_proj_weight"] = inp[pre + "self_attn.in_proj.weight"]
            st[pre + "self_attn.in_proj_bias"] = inp[pre + "self_attn.in_proj.bias"]
            st.update(lin(pre + "self_attn.out_proj", d, d))
            st.update(lin(pre + "linear1", ffn, d))
            st.update(lin(pre + "linear2", d, ffn))
            for nm in ("norm1", "norm2"):
                st[pre + nm + ".weight"] = torch.ones(d)
                st[pre + nm + ".bias"] = torch.zeros(d)
        st["norm.weight"], st["norm.bias"] = torch.ones(d), torch.zeros(d)
        st.update(lin("head.0", d, d))
        st.update(lin("head.2", outputs, d))
        return {k: v.to(torch.bfloat16).float() for k, v in st.items()}

    def new_cache(self, rows: int, slots: int = MAX_EVENTS + 2) -> SeqKVCache:
        return SeqKVCache(self, rows, slots)

    # -- tokens --------------------------------------------------------------------
    def start_token(self, start: torch.Tensor, seat: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """SeqNet.start_token (python/cugo_seq50.py:271-274): fp32 [n, d];
        row i reads start[i % len(start)]."""
        return self.ext.start_embed(start, seat, self.start_wt, self.start_b, self.position[0],
                                    self.token_type[0], out=out)

    def event_token(self, words: torch.Tensor, seat: torch.Tensor, index: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """SeqNet.event_token (python/cugo_seq50.py:276-282): fp32 [n, d] for n =
        len(seat); row i reads words[i % len(words)] and index[i % len(words)]."""
        return self.ext.event_embed(words, seat, index, self.event_wt, self.event_b, self.position,
                                    self.token_type[1], out=out)

    def query_token(self, query: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """SeqNet.query_token (python/cugo_seq50.py:284-286) from the bf16 [n, 904]
        query input that observe_query_bf16 writes: fp32 [n, d]."""
        h = self.ext.linear(query, self.q_w0, self.q_b0, act=ACT_GELU)
        return self.ext.linear(h, self.q_w1, self.q_b1, out=out, out_dtype=torch.float32)

    # -- decode --------------------------------------------------------------------
    def cached_step(self, cache: SeqKVCache, x: torch.Tensor, slots: int | None = None,
                    rows: torch.Tensor | None = None) -> torch.Tensor:
        """SeqNet.cached_step (python/cugo_seq50.py:291-322) on x fp32 [n, d], updated
        in place and returned.  Token i goes to slot min(cache.length[row], slots - 1)
        of its cache row (rows[i], default i) and attends slots 0.. that one."""
        ext = self.ext
        n, d = x.shape
        heads, dh = self.heads, d // self.heads
        t = cache.slots if slots is None else min(slots, cache.slots)
        for i, L in enumerate(self.blocks):
            a = ext.layernorm(x, L.norm1_w, L.norm1_b, self.eps)
            qkv = ext.linear(a, L.w_in, L.b_in)
            q = qkv[:, :d].view(n, heads, dh)
            k = qkv[:, d:2 * d].view(n, heads, dh)
            v = qkv[:, 2 * d:].view(n, heads, dh)
            att = ext.decode_attention(q, cache.k[i], cache.v[i], cache.length, rows=rows, k_new=k,
                                       v_new=v, pos_clamp=t - 1)
            ext.linear(att.view(n, d), L.w_out, L.b_out, residual=x, out=x)
            a = ext.layernorm(x, L.norm2_w, L.norm2_b, self.eps)
            f = ext.linear(a, L.w1, L.b1, act=ACT_GELU)
            ext.linear(f, L.w2, L.b2, residual=x, out=x)
        return x

    def cached_step_segments(self, cache: SeqKVCache, x: torch.Tensor,
                             segments: list[tuple], active: torch.Tensor | None = None
                             ) -> torch.Tensor:
        """cached_step over consecutive row segments of x fp32 [n, d] (updated in place
        and returned) that share every layer's LayerNorm and GEMM launches.  segments =
        [(count, rows, positions)]: the segment's tokens go to cache rows `rows`
        (default 0..count-1) at slot min(positions[row], slots - 1).  With `active`
        (bool [n]) only those tokens attend and append (the others' outputs are
        meaningless and must not be used).  At every layer the
        segments' attention launches (each with its KV append) run in order, so a later
        segment sees the slots an earlier one appended exactly as if it had run as its
        own pass after it; every other layer computes each row on its own, so each
        row's result is cached_step's."""
        ext = self.ext
        n, d = x.shape
        heads, dh = self.heads, d // self.heads
        if sum(c for c, _, _ in segments) != n:
            raise ValueError("the segments must cover the rows of x")
        clamp = cache.slots - 1
        att = torch.empty((n, d), dtype=torch.bfloat16, device=x.device)
        for i, L in enumerate(self.blocks):
            a = ext.layernorm(x, L.norm1_w, L.norm1_b, self.eps)
            qkv = ext.linear(a, L.w_in, L.b_in)
            q = qkv[:, :d].view(n, heads, dh)
            k = qkv[:, d:2 * d].view(n, heads, dh)
            v = qkv[:, 2 * d:].view(n, heads, dh)
            s0 = 0
            for count, rows, positions in segments:
                s1 = s0 + count
                ext.decode_attention(q[s0:s1], cache.k[i], cache.v[i], positions, rows=rows,
                                     k_new=k[s0:s1], v_new=v[s0:s1], pos_clamp=clamp,
                                     out=att[s0:s1].view(count, heads, dh),
                                     active=None if active is None else active[s0:s1])
                s0 = s1
            ext.linear(att, L.w_out, L.b_out, residual=x, out=x)
            a = ext.layernorm(x, L.norm2_w, L.norm2_b, self.eps)
            f = ext.linear(a, L.w1, L.b1, act=ACT_GELU)
            ext.linear(f, L.w2, L.b2, residual=x, out=x)
        return x

    # -- training forward over whole games ---------------------------------------
    def forward_games(self, hist, features: torch.Tensor, legal: torch.Tensor,
                      seen: torch.Tensor, length: int | None = None) -> torch.Tensor:
        """SeqNet.forward_games (python/cugo_seq50.py:240-265): every decision of each
        (game, seat) sequence at once.  hist has .events int64 [S, MAX_EVENTS, 9],
        .count [S] (the game's events), .start [S, 8], .seat [S]; features [S, Q, 720],
        legal [S, Q, 179], seen int64 [S, Q] (events visible at each decision).
        Returns fp32 [S, Q, outputs].

        Token rows live in three blocks — S openings, S x L events, S x Q queries —
        embedded straight into the fp32 residual stream by the start/event gather-sum
        kernels and the query MLP; each layer is LayerNorm, the QKV GEMM, the games
        attention kernel (opening, causal events, queries over their visible events
        and themselves), the out-projection and FFN GEMMs with the residual in their
        epilogues; the head reads the query rows only."""
        ext, d = self.ext, self.d_model
        s_n, q_n = seen.shape
        L = max(1, int(hist.count.max())) if length is None else max(1, length)
        if L > MAX_EVENTS:
            raise ValueError(f"length {L} exceeds {MAX_EVENTS} events")
        dev = self.device
        n_ev, n_q = s_n * L, s_n * q_n
        x = torch.empty((s_n + n_ev + n_q, d), dtype=torch.float32, device=dev)
        seat = hist.seat.to(dev, torch.int64).contiguous()
        self.start_token(hist.start.to(dev).contiguous(), seat, out=x[:s_n])
        if n_ev:
            words = hist.events[:, :L].to(dev).reshape(n_ev, self.ext.EVENT_WORDS).contiguous()
            index = torch.arange(L, device=dev).repeat(s_n)
            self.event_token(words, seat.repeat_interleave(L), index, out=x[s_n:s_n + n_ev])
        if n_q:
            query = torch.zeros((n_q, QUERY_LD), dtype=torch.bfloat16, device=dev)
            query[:, :FEATURES] = features.reshape(n_q, FEATURES)
            query[:, FEATURES:QUERY_IN] = legal.reshape(n_q, ACTIONS)
            self.query_token(query, out=x[s_n + n_ev:])
        seen_flat = seen.to(dev, torch.int64).reshape(-1).contiguous()
        for blk in self.blocks:
            a = ext.layernorm(x, blk.norm1_w, blk.norm1_b, self.eps)
            qkv = ext.linear(a, blk.w_in, blk.b_in)
            att = ext.games_attention(qkv, s_n, L, q_n, seen_flat)
            ext.linear(att, blk.w_out, blk.b_out, residual=x, out=x)
            a = ext.layernorm(x, blk.norm2_w, blk.norm2_b, self.eps)
            f = ext.linear(a, blk.w1, blk.b1, act=ACT_GELU)
            ext.linear(f, blk.w2, blk.b2, residual=x, out=x)
        return self.readout(x[s_n + n_ev:]).reshape(s_n, q_n, self.outputs)

    def readout(self, h: torch.Tensor) -> torch.Tensor:
        """SeqNet.readout (python/cugo_seq50.py:288-289, head(norm(h))): fp32 [n, outputs]."""
        a = self.ext.layernorm(h, self.norm_w, self.norm_b, self.eps)
        z = self.ext.linear(a, self.h_w0, self.h_b0, act=ACT_GELU)
        out = torch.empty((h.shape[0], self.out_ld), dtype=torch.float32, device=h.device)
        self.ext.linear(z, self.h_w1, self.h_b1, out=out[:, :self.outputs])
        return out[:, :self.outputs]
