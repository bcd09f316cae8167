"""GPU: the policy forward that allocates nothing, through the C ABI.

Some callers of this library cannot allocate device memory on their hot path — a
serving process in another language that hands over only its own input and output
buffers, or a runtime that reserved all device memory at start-up.  For them
cugo_b200_policy_forward_noalloc keeps the hidden activations in a buffer compiled
into the library.  This test calls it directly with ctypes and checks its logits
against the regular policy forward (ResidualMlpPolicy, which allocates its
activations with torch) on two calls in a row with different batches, so stale
contents of the shared buffer would show, and checks that an oversized batch is
refused.  The regular forward is taken on its layer-per-launch path
(CUGO_B200_MLP_FUSED=0), which runs the same GEMM kernels in the same order, so the
tolerance is the GEMM tests' single-layer bound, 1% relative + 1e-2 absolute.

Collected last (file name) so a first-failure stop has already run the rest.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
CAPACITY = 4 << 20  # rows x hidden of the built-in buffer
ERR_CAPACITY = -4


def _entry():
    from cugo_b200 import load_library

    fn = load_library().cugo_b200_policy_forward_noalloc
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    fn.argtypes = [vp, i64, i64, i64, i64, i32, i64, vp, vp, i32, vp, i64, vp, vp]
    fn.restype = ctypes.c_int
    return fn


def _policy():
    from cugo_b200.policy import ResidualMlpPolicy

    pol = ResidualMlpPolicy(512, 3, "relu", device=DEV, seed=3)
    g = torch.Generator().manual_seed(4)
    pol.biases = [(torch.randn(b.shape, generator=g) * 0.05).to(DEV, torch.bfloat16)
                  for b in pol.biases]
    return pol


def _noalloc(fn, pol, x):
    m = x.size(0)
    layers = len(pol.weights)
    weights = (ctypes.c_void_p * layers)(*[w.data_ptr() for w in pol.weights])
    biases = (ctypes.c_void_p * layers)(*[b.data_ptr() for b in pol.biases])
    out = torch.full((m, 180), float("nan"), dtype=torch.float32, device=DEV)
    error = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = fn(x.data_ptr(), x.stride(0), m, x.size(1), pol.hidden, pol.blocks, pol.outputs,
            ctypes.cast(weights, ctypes.c_void_p), ctypes.cast(biases, ctypes.c_void_p), 1,
            out.data_ptr(), out.stride(0), error.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, out, int(error.item())


def test_noalloc_forward_matches_policy_on_consecutive_calls(monkeypatch):
    monkeypatch.setenv("CUGO_B200_MLP_FUSED", "0")
    fn = _entry()
    pol = _policy()
    g = torch.Generator().manual_seed(5)
    for m in (4096, 1000):  # the second, smaller call must not see the first's rows
        x = torch.randn((m, 720), generator=g).to(DEV, torch.bfloat16)
        expect = pol(x)
        rc, got, err = _noalloc(fn, pol, x)
        assert rc == 0 and err == 0
        diff = (got - expect).abs()
        assert bool((diff <= 1e-2 * expect.abs() + 1e-2).all()), float(diff.max())


def test_noalloc_forward_refuses_oversized_batch():
    fn = _entry()
    pol = _policy()
    m = CAPACITY // pol.hidden + 1
    x = torch.zeros((m, 720), dtype=torch.bfloat16, device=DEV)
    rc, out, _ = _noalloc(fn, pol, x)
    assert rc == ERR_CAPACITY
    assert bool(torch.isnan(out).all())  # nothing was written
