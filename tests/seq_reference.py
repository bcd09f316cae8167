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
