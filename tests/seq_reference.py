"""Test-side restatements for the sequence policy's decode path (test infrastructure).

decode_attention_fp32 restates the reference's matrix-product path of
decode_attention (python/cugo_seq_attention50.py:58-62) in fp32: gather the cache
rows, score slots 0..pos with q.k * dh^-0.5, softmax, weight the values.  It is
pinned against the reference function itself by tests/golden/seq_decode.npz.

attention_case and history_case build seeded inputs from a CPU torch.Generator,
so the golden script and the tests draw identical tensors without storing them.
"""
from __future__ import annotations

import torch

HEADS, DH = 8, 32


def attention_case(seed: int, n: int, n_rows: int, slots: int = 50, heads: int = HEADS,
                   dh: int = DH):
    """q [n, heads, dh], keys/values [n_rows, heads, slots, dh] (bf16-valued fp32),
    pos [n] in [0, slots), rows [n] distinct when n <= n_rows."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((n, heads, dh), generator=g).to(torch.bfloat16).float()
    keys = torch.randn((n_rows, heads, slots, dh), generator=g).to(torch.bfloat16).float()
    values = torch.randn((n_rows, heads, slots, dh), generator=g).to(torch.bfloat16).float()
    pos = torch.randint(0, slots, (n,), generator=g)
    pos[: min(n, 4)] = torch.tensor([0, slots - 1, 31, 32])[: min(n, 4)].clamp_max(slots - 1)
    if n <= n_rows:
        rows = torch.randperm(n_rows, generator=g)[:n]
    else:
        rows = torch.randint(0, n_rows, (n,), generator=g)
    return q, keys, values, pos, rows


def decode_attention_fp32(q, keys, values, pos, rows):
    """fp32 decode attention: [n, heads, dh]."""
    n, heads, dh = q.shape
    slots = keys.shape[2]
    k = keys.index_select(0, rows).float()
    v = values.index_select(0, rows).float()
    mask = torch.arange(slots, device=q.device).view(1, 1, 1, slots) <= pos.view(n, 1, 1, 1)
    scores = torch.matmul(q.float().unsqueeze(2), k.transpose(-1, -2)) * dh ** -0.5
    probs = torch.softmax(scores.masked_fill(~mask, float("-inf")), -1)
    return torch.matmul(probs, v).squeeze(2)


def query_input(features: torch.Tensor, legal: torch.Tensor, width: int = 904) -> torch.Tensor:
    """The hybrid query input cat(features, legal) as bf16 rows padded to `width`."""
    n = features.shape[0]
    out = torch.zeros((n, width), dtype=torch.bfloat16, device=features.device)
    out[:, :720] = features.to(torch.bfloat16)
    out[:, 720:899] = legal.to(torch.bfloat16)
    return out


# ---- the training forward over whole games (python/cugo_seq50.py:91-128, 200-265) ----

def _planes(masks: torch.Tensor, width: int = 50) -> torch.Tensor:
    """[..., width] 0/1 float planes of the low `width` bits of int64 masks."""
    shifts = torch.arange(width, device=masks.device)
    return ((masks.unsqueeze(-1) >> shifts) & 1).float()


def event_tokens(events: torch.Tensor, seat: torch.Tensor, length: int) -> torch.Tensor:
    """Observer-relative event tokens [B, length, 414] (fp32): eight card planes
    (played, own draws, flipped, my gain, their gain, my loss, their loss, shown),
    the kind one-hot clamped to 11, the "mine" flag and the opponent's draw count."""
    ev = events[:, :length]
    sv = seat.view(-1, 1)
    mine = (ev[..., 8] & 0xFF) == sv
    kind = ((ev[..., 8] >> 8) & 0xFF).clamp_max(11)
    s0 = sv == 0
    pick = lambda a, b: torch.where(s0, ev[..., a], ev[..., b])  # noqa: E731
    slots = [ev[..., 0], torch.where(mine, ev[..., 1], torch.zeros_like(ev[..., 1])), ev[..., 2],
             pick(3, 4), pick(4, 3), pick(5, 6), pick(6, 5), ev[..., 7]]
    drawn = torch.where(mine, torch.zeros_like(kind), _planes(ev[..., 1]).sum(-1).long())
    onehot = torch.nn.functional.one_hot(kind, 12).float()
    return torch.cat([_planes(m) for m in slots] + [onehot, mine.float().unsqueeze(-1),
                                                    drawn.float().unsqueeze(-1)], -1)


def start_tokens(start: torch.Tensor, seat: torch.Tensor) -> torch.Tensor:
    """Opening tokens [B, 274] (fp32): hand, floor, my and their captures, mission
    cards, 12 neutral months, mission type one-hot (clamped to 7), multiplier / 4,
    "I move first", my and their multi / 8."""
    s0 = seat == 0
    side = lambda a, b: torch.where(s0, start[:, a], start[:, b])  # noqa: E731
    planes = _planes(torch.stack((side(0, 1), start[:, 2], side(3, 4), side(4, 3), start[:, 5]), -1))
    head = start[:, 7]
    mine_multi = torch.where(s0, (head >> 24) & 0xFF, (head >> 32) & 0xFF)
    their_multi = torch.where(s0, (head >> 32) & 0xFF, (head >> 24) & 0xFF)
    scal = torch.stack((((head >> 8) & 0xFF).float() / 4.0, (((head >> 16) & 1) == seat).float(),
                        mine_multi.float() / 8.0, their_multi.float() / 8.0), -1)
    return torch.cat((planes.flatten(-2), _planes(start[:, 6], 12),
                      torch.nn.functional.one_hot((head & 0xFF).clamp_max(7), 8).float(), scal), -1)


def forward_games(p: dict, events, count, start, seat, features, legal, seen, length: int,
                  heads: int = HEADS) -> torch.Tensor:
    """SeqNet.forward_games with state dict p (hybrid mode) in plain torch: tokens
    [opening, length events, one query per decision]; the opening sees itself,
    events are causal, a query sees the opening, its visible events and itself;
    pre-LN layers (GELU FFN), then LayerNorm and the head on the query rows."""
    f = torch.nn.functional
    s_n, q_n = seen.shape
    d = p["position"].shape[1]
    lin = lambda x, n: f.linear(x, p[n + ".weight"], p[n + ".bias"])  # noqa: E731
    x0 = lin(start_tokens(start, seat), "start_in") + p["position"][0] + p["token_type"][0]
    xe = lin(event_tokens(events, seat, length), "event_in") + p["position"][1:length + 1] \
        + p["token_type"][1]
    xq = lin(f.gelu(lin(torch.cat((features.float(), legal.float()), -1), "query_in.0")),
             "query_in.2") + p["token_type"][2]
    x = torch.cat((x0.unsqueeze(1), xe, xq), 1)
    t = 1 + length + q_n
    allowed = torch.zeros(s_n, t, t, dtype=torch.bool, device=x.device)
    allowed[:, :, 0] = True
    allowed[:, 1:length + 1, 1:length + 1] = torch.ones(length, length, dtype=torch.bool,
                                                        device=x.device).tril()
    allowed[:, length + 1:, 1:length + 1] = torch.arange(length, device=x.device).view(1, 1, -1) \
        < seen.unsqueeze(-1)
    allowed[:, length + 1:, length + 1:] = torch.eye(q_n, dtype=torch.bool, device=x.device)
    dh = d // heads
    for i in range(len({k.split(".")[2] for k in p if k.startswith("encoder.layers.")})):
        pre = f"encoder.layers.{i}."
        a = f.layer_norm(x, (d,), p[pre + "norm1.weight"], p[pre + "norm1.bias"])
        qkv = f.linear(a, p[pre + "self_attn.in_proj_weight"], p[pre + "self_attn.in_proj_bias"])
        q, k, v = (z.reshape(s_n, t, heads, dh).transpose(1, 2) for z in qkv.chunk(3, -1))
        sc = (q @ k.transpose(-1, -2)) * dh ** -0.5
        att = torch.softmax(sc.masked_fill(~allowed.unsqueeze(1), float("-inf")), -1) @ v
        x = x + lin(att.transpose(1, 2).reshape(s_n, t, d), pre + "self_attn.out_proj")
        a = f.layer_norm(x, (d,), p[pre + "norm2.weight"], p[pre + "norm2.bias"])
        x = x + lin(f.gelu(lin(a, pre + "linear1")), pre + "linear2")
    h = f.layer_norm(x[:, length + 1:], (d,), p["norm.weight"], p["norm.bias"])
    return lin(f.gelu(lin(h, "head.0")), "head.2")
