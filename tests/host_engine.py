"""ctypes view of the host build of the engine headers (tests/native/engine_host.cpp).

Used by the CPU test suite to compare the engine's rule code with the oracle without a
GPU.  The build goes to tests/_build/ (git-ignored).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "native" / "engine_host.cpp"
HEADERS = sorted((ROOT / "cugo_b200" / "csrc" / "engine").glob("*.cuh"))
LIB = ROOT / "tests" / "_build" / "libcugo_engine_host.so"

STATE_BYTES, FEATURES, ACTIONS, EVENT_WORDS, START_WORDS = 248, 720, 179, 9, 8
_lib = None


def build() -> Path:
    newest = max(p.stat().st_mtime for p in [SRC, *HEADERS])
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        LIB.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", str(SRC), "-o", str(LIB)],
                       check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def create(seeds, first):
    seeds = np.ascontiguousarray(seeds, dtype=np.int64)
    first = np.ascontiguousarray(first, dtype=np.int64)
    rows = np.zeros((seeds.shape[0], STATE_BYTES), dtype=np.uint8)
    lib().cugo_host_create(_p(seeds), _p(first), ctypes.c_int64(seeds.shape[0]), _p(rows))
    return rows


def observe(rows):
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    n = rows.shape[0]
    features = np.zeros((n, FEATURES), dtype=np.float32)
    legal = np.zeros((n, ACTIONS), dtype=np.uint8)
    player = np.zeros(n, dtype=np.uint8)
    done = np.zeros(n, dtype=np.uint8)
    status = np.zeros(n, dtype=np.int16)
    lib().cugo_host_observe(_p(rows), ctypes.c_int64(n), _p(features), _p(legal), _p(player),
                            _p(done), _p(status))
    return features, legal.astype(bool), player, done.astype(bool), status


def step(rows, actions, events: bool = False):
    rows = np.array(rows, dtype=np.uint8, order="C", copy=True)
    actions = np.ascontiguousarray(actions, dtype=np.int64)
    n = rows.shape[0]
    reward = np.zeros(n, dtype=np.float32)
    done = np.zeros(n, dtype=np.uint8)
    nagari = np.zeros(n, dtype=np.uint8)
    status = np.zeros(n, dtype=np.int16)
    committed = np.zeros(n, dtype=np.uint8)
    ev = np.zeros((n, EVENT_WORDS), dtype=np.int64)
    lib().cugo_host_step(_p(rows), _p(actions), ctypes.c_int64(n), _p(reward), _p(done), _p(nagari),
                         _p(status), _p(committed), _p(ev))
    out = (rows, reward, done.astype(bool), nagari.astype(bool), status, committed.astype(bool))
    return out + (ev,) if events else out


def legal_check(rows):
    """Per row, the first action (0..255) on which the step's single-action legality
    check disagrees with the primary legal mask, or -1."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.zeros(rows.shape[0], dtype=np.int32)
    lib().cugo_host_legal_check(_p(rows), ctypes.c_int64(rows.shape[0]), _p(out))
    return out


def start(rows):
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.zeros((rows.shape[0], START_WORDS), dtype=np.int64)
    lib().cugo_host_start(_p(rows), ctypes.c_int64(rows.shape[0]), _p(out))
    return out


def stock(rows):
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.zeros(rows.shape[0], dtype=np.int64)
    lib().cugo_host_stock(_p(rows), ctypes.c_int64(rows.shape[0]), _p(out))
    return out
