"""The C ABI library loads, exports every declared entry point and validates its
arguments on the host (CPU only: no call here reaches a kernel launch)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from cugo_b200 import ext as ext_mod
from cugo_b200 import load_library

HEADER = Path(__file__).resolve().parents[1] / "include" / "cugo_b200.h"


def declared_symbols() -> list[str]:
    return re.findall(r"CUGO_B200_API\s+\w+\s+(cugo_b200_\w+)\s*\(", HEADER.read_text())


def test_library_exports_every_declared_symbol():
    lib = load_library()
    names = declared_symbols()
    assert len(names) >= 24
    for name in names:
        assert hasattr(lib, name), name


def test_contract_constants():
    e = ext_mod.CugoB200Extension(load_library())
    assert (e.FEATURE_COUNT, e.ACTION_COUNT, e.PRIMARY_ACTION_COUNT, e.CHOICE_ACTION_BEGIN,
            e.EVENT_WORDS, e.START_WORDS, e.STATE_BYTES, e.STATUS_OK) == (720, 179, 127, 127, 9, 8,
                                                                           248, 0)
    assert load_library().cugo_b200_abi_version() == 1


def test_argument_errors_without_launch():
    lib = load_library()
    # Negative sizes and missing pointers are rejected before any launch.
    assert lib.cugo_b200_create(None, None, -1, None, None) == -1
    assert lib.cugo_b200_create(None, None, 4, None, None) == -1
    assert lib.cugo_b200_observe(None, -2, None, None, None, None, None, None) == -1
    assert lib.cugo_b200_step_indexed(None, 4, None, None, 2, None, None, None, None, None,
                                      None) == -1
    # Misaligned states pointer.
    assert lib.cugo_b200_create(8, 8, 1, 0x1003, None) == -2
    # Empty batches are a no-op success.
    assert lib.cugo_b200_create(None, None, 0, None, None) == 0
    assert lib.cugo_b200_clone_indexed(None, 0, None, 0, None, None) == 0
    assert lib.cugo_b200_start(None, 0, None, None) == 0


@pytest.fixture()
def cpu_ext():
    return ext_mod.CugoB200Extension(load_library())


def test_shim_messages_match_reference(cpu_ext):
    e = cpu_ext
    ids = torch.zeros(2, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="seeds must be a CUDA tensor"):
        e.create(ids, ids)
    with pytest.raises(RuntimeError, match="states must be a CUDA tensor"):
        e.observe(torch.zeros((2, 248), dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="states must be a CUDA tensor"):
        e.step_indexed(torch.zeros((2, 248), dtype=torch.uint8), ids, ids)


def test_loader_requires_cuda(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    monkeypatch.setattr(ext_mod, "_EXT", None)
    with pytest.raises(RuntimeError, match="PyTorch CUDA is not available"):
        ext_mod.load_extension()


def test_noalloc_forward_capacity_check_does_not_wrap():
    """Sizes whose product wraps a 64-bit integer (2^33 rows x 2^31 hidden) are
    refused as over capacity before anything is read or launched, like any batch
    larger than the built-in activation buffer."""
    fn = load_library().cugo_b200_policy_forward_noalloc
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    fn.argtypes = [vp, i64, i64, i64, i64, i32, i64, vp, vp, i32, vp, i64, vp, vp]
    fn.restype = ctypes.c_int
    weights = (ctypes.c_void_p * 8)(*([0x1000] * 8))
    w = ctypes.cast(weights, ctypes.c_void_p)
    err_capacity = -4
    for m, hidden in ((1 << 33, 1 << 31), (1 << 62, 4), (1, (4 << 20) + 1), ((4 << 20) // 512 + 1, 512)):
        assert fn(None, 720, m, 720, hidden, 3, 180, w, None, 1, None, 180, None, None) == err_capacity


def test_wgrad_arguments_checked_before_launch():
    """The weight-gradient entry refuses bad sizes, misaligned operands and a scratch
    buffer smaller than its own size query before touching the device; the query
    covers every split's padded partial tile."""
    lib = load_library()
    fn = lib.cugo_b200_wgrad_bf16
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    fn.argtypes = [vp, i64, vp, i64, i64, i64, i64, vp, i64, vp, i64, vp, vp]
    fn.restype = ctypes.c_int
    q = lib.cugo_b200_wgrad_scratch_floats
    q.argtypes, q.restype = [i64, i64, i64], i64
    need = q(32768, 512, 512)
    assert need > 0 and need % (512 * 512) == 0  # whole 128 x 256 tiles per split
    assert q(32768, 179, 512) % (256 * 512) == 0  # 179 outputs padded to two 128-row tiles
    assert q(0, 512, 512) == 0
    a = 0x10000
    assert fn(a, 512, a, 512, 64, 0, 512, a, 512, a, need, None, None) == -1   # no outputs
    assert fn(a, 100, a, 512, 64, 512, 512, a, 512, a, need, None, None) == -1  # lddy < n_out
    assert fn(a + 8, 512, a, 512, 64, 512, 512, a, 512, a, need, None, None) == -2
    assert fn(a, 516, a, 512, 64, 512, 512, a, 512, a, need, None, None) == -2  # stride not 16 B
    small = q(64, 512, 512) - 1
    assert fn(a, 512, a, 512, 64, 512, 512, a, 512, a, small, None, None) == -4
    assert fn(a, 512, a, 512, 64, 512, 512, a, 512, None, need, None, None) == -4


def test_running_init_arguments_checked_before_launch():
    """The running-set entry refuses a negative size, missing outputs and a scratch
    buffer shorter than its own size query before touching the device."""
    lib = load_library()
    fn = lib.cugo_b200_running_init
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    fn.argtypes = [vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, i64, vp]
    fn.restype = ctypes.c_int
    q = lib.cugo_b200_running_init_scratch
    q.argtypes, q.restype = [i64], i64
    assert q(0) == 0 and q(1) == 2 and q(64) == 4 and q(65) == 6 and q(-1) == -1
    a = 0x10000
    assert fn(a, -1, a, a, a, a, a, a, a, a, 4, None) == -1        # negative size
    assert fn(a, 64, None, a, a, a, a, a, a, a, 4, None) == -1     # no ids
    assert fn(a, 64, a, a, a, a, a, a, None, a, 4, None) == -1     # no bad counter
    assert fn(a, 65, a, None, a, a, a, a, a, a, q(65) - 1, None) == -4  # scratch too short
