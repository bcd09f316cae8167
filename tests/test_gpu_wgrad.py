"""GPU parity: the tcgen05 weight-gradient kernel (cugo_b200_wgrad_bf16, split over
the rows) against the fp32 product of the same bf16 operands."""
from __future__ import annotations

import pytest
import torch

from cugo_b200 import load_extension

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _operands(rows, n_out, n_in, ld_out, ld_in, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    dy = torch.zeros((rows, ld_out), dtype=torch.bfloat16)
    x = torch.zeros((rows, ld_in), dtype=torch.bfloat16)
    dy[:, :n_out] = torch.randn((rows, n_out), generator=g).to(torch.bfloat16)
    x[:, :n_in] = torch.randn((rows, n_in), generator=g).to(torch.bfloat16)
    # Padding columns hold junk: the kernel must not read them into the result.
    dy[:, n_out:] = 7.0
    x[:, n_in:] = -3.0
    return dy.to(DEV), x.to(DEV)


@pytest.mark.parametrize("rows,n_out,n_in,ld_out,ld_in", [
    (32768, 512, 512, 512, 512),      # a hidden layer of a 3x512 update minibatch
    (32768, 179, 512, 184, 512),      # the actor head (dy rows padded to 16 bytes)
    (32768, 512, 770, 512, 776),      # the critic's input layer
    (32768, 512, 720, 512, 720),      # the actor's input layer
    (4097, 2048, 2048, 2048, 2048),   # 4x2048 hidden layer, ragged rows
    (100, 64, 40, 64, 40),            # fewer rows than one 64-row stage
    (1, 8, 8, 8, 8),
])
def test_wgrad_matches_fp32(rows, n_out, n_in, ld_out, ld_in):
    ext = load_extension()
    dy, x = _operands(rows, n_out, n_in, ld_out, ld_in, seed=rows + n_out)
    out = torch.full((n_out, n_in), float("nan"), dtype=torch.float32, device=DEV)
    ext.wgrad_bf16(dy, x, out, n_out=n_out, n_in=n_in)
    ref = dy[:, :n_out].float().t() @ x[:, :n_in].float()
    scale = float(ref.abs().max())
    err = float((out - ref).abs().max())
    # fp32 accumulation of exact bf16 products in another order.
    assert err <= 2e-5 * scale + 1e-5, (err, scale)
    again = torch.empty_like(out)
    ext.wgrad_bf16(dy, x, again, n_out=n_out, n_in=n_in)
    assert torch.equal(out, again)  # the splits are added in a fixed order


def test_wgrad_into_a_strided_gradient():
    """dw with a row stride wider than n_in (a view into a larger buffer): only the
    n_in columns of each row are written."""
    ext = load_extension()
    dy, x = _operands(2048, 256, 200, 256, 200, seed=3)
    big = torch.full((256, 264), 5.0, dtype=torch.float32, device=DEV)
    ext.wgrad_bf16(dy, x, big[:, :200])
    ref = dy.float().t() @ x.float()
    assert float((big[:, :200] - ref).abs().max()) <= 2e-5 * float(ref.abs().max()) + 1e-5
    assert bool((big[:, 200:] == 5.0).all())
