"""CPU: host-side argument checks of the fused policy step and the round tail
(cugo_b200_mlp_fused, cugo_b200_mlp_fused_sample, cugo_b200_step_compact).  Every call
here returns before any CUDA call: fake, never dereferenced device pointers."""
from __future__ import annotations

import ctypes

from cugo_b200 import load_library

ERR_ARG, ERR_ALIGN, OK = -1, -2, 0
P = 0x10000  # a 16-byte aligned fake device pointer


def _weights(layers: int):
    return (ctypes.c_void_p * layers)(*([P] * layers))


def _fused(lib, m=1000, k_in=720, blocks=3, n_out=180, x=P, ldx=720, out=P, ldo=180):
    return lib.cugo_b200_mlp_fused(x, ldx, m, k_in, blocks, _weights(2 + 2 * blocks), None,
                                   n_out, 1, out, ldo, None, None)


def _sample(lib, m=1000, n_out=180, legal=P, rows=None, n_games=0, actions=P, logp=P):
    return lib.cugo_b200_mlp_fused_sample(P, 720, m, 720, 3, _weights(8), None, n_out, 1, legal,
                                          P, P, rows, n_games, 12345, 0, actions, logp, None, 0,
                                          None, None, None)


def test_mlp_fused_rejects_bad_shapes_before_launch():
    lib = load_library()
    assert _fused(lib, m=0) == OK                 # an empty batch is a no-op
    assert _fused(lib, m=-1) == ERR_ARG
    assert _fused(lib, k_in=1032, ldx=1032) == ERR_ARG  # K above 1,024
    assert _fused(lib, blocks=5) == ERR_ARG       # more than 4 blocks
    assert _fused(lib, n_out=257, ldo=260) == ERR_ARG  # more than 256 outputs
    assert _fused(lib, ldx=700) == ERR_ARG        # row stride below K
    assert _fused(lib, out=None) == ERR_ARG       # no output and no sampling
    assert _fused(lib, x=P + 8) == ERR_ALIGN      # x not 16-byte aligned
    assert _fused(lib, k_in=724, ldx=728) == ERR_ALIGN  # K not a multiple of 8


def test_mlp_fused_sample_rejects_bad_arguments_before_launch():
    lib = load_library()
    assert _sample(lib, m=0) == OK
    assert _sample(lib, actions=None) == ERR_ARG
    assert _sample(lib, logp=None) == ERR_ARG
    assert _sample(lib, n_out=178) == ERR_ARG     # fewer outputs than actions
    assert _sample(lib, legal=P + 4) == ERR_ALIGN  # legal words not 8-byte aligned
    assert _sample(lib, rows=P, n_games=-1) == ERR_ARG


def test_step_compact_rejects_a_count_it_would_overwrite():
    lib = load_library()
    # The running count read by the kernels cannot be the one the call rewrites.
    rc = lib.cugo_b200_step_compact(P, 100, P, P, 10, P, P, P, P, P, P + 64, P + 128, P + 64, None)
    assert rc == ERR_ARG
    assert lib.cugo_b200_step_compact(P, 100, None, P, 10, P, P, P, P, P, P, P, None, None) == ERR_ARG
    assert lib.cugo_b200_step_compact(P, -1, P, P, 10, P, P, P, P, P, P, P, None, None) == ERR_ARG
