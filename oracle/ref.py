"""ctypes view of oracle/_ref/libcugo_ref.so (TEST INFRASTRUCTURE ONLY).

The library is the reference's own header-only engine compiled from its sources by
oracle/Makefile (see oracle/ref_harness.cpp for the reference functions each entry
point runs).  Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline may
use this module; the product never does.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "libcugo_ref.so"

STATE_BYTES = 248
FEATURES = 720
ACTIONS = 179
EVENT_WORDS = 9
START_WORDS = 8

_lib = None


def available() -> bool:
    return LIB_PATH.is_file()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            raise RuntimeError(f"oracle library missing: {LIB_PATH} (run `make -C oracle`)")
        _lib = ctypes.CDLL(str(LIB_PATH))
        if _lib.cugo_ref_state_bytes() != STATE_BYTES:
            raise RuntimeError("oracle TorchEnv50 size mismatch")
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def create(seeds: np.ndarray, first: np.ndarray, threads: int | None = None) -> np.ndarray:
    seeds = np.ascontiguousarray(seeds, dtype=np.int64)
    first = np.ascontiguousarray(first, dtype=np.int64)
    n = seeds.shape[0]
    rows = np.zeros((n, STATE_BYTES), dtype=np.uint8)
    lib().cugo_ref_create(_p(seeds), _p(first), ctypes.c_int64(n), _p(rows),
                          ctypes.c_int(threads or default_threads()))
    return rows


def canonicalize(rows: np.ndarray) -> np.ndarray:
    rows = np.array(rows, dtype=np.uint8, order="C", copy=True)
    lib().cugo_ref_canonicalize(_p(rows), ctypes.c_int64(rows.shape[0]))
    return rows


def observe(rows: np.ndarray, threads: int | None = None):
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    n = rows.shape[0]
    features = np.zeros((n, FEATURES), dtype=np.float32)
    legal = np.zeros((n, ACTIONS), dtype=np.uint8)
    player = np.zeros(n, dtype=np.uint8)
    done = np.zeros(n, dtype=np.uint8)
    status = np.zeros(n, dtype=np.int16)
    lib().cugo_ref_observe(_p(rows), ctypes.c_int64(n), _p(features), _p(legal), _p(player),
                           _p(done), _p(status), ctypes.c_int(threads or default_threads()))
    return features, legal.astype(bool), player, done.astype(bool), status


def step(rows: np.ndarray, actions: np.ndarray, threads: int | None = None, events: bool = False):
    """Steps a COPY of rows; returns (new_rows, reward, done, nagari, status, committed[, events])."""
    rows = np.array(rows, dtype=np.uint8, order="C", copy=True)
    actions = np.ascontiguousarray(actions, dtype=np.int64)
    n = rows.shape[0]
    reward = np.zeros(n, dtype=np.float32)
    done = np.zeros(n, dtype=np.uint8)
    nagari = np.zeros(n, dtype=np.uint8)
    status = np.zeros(n, dtype=np.int16)
    committed = np.zeros(n, dtype=np.uint8)
    ev = np.zeros((n, EVENT_WORDS), dtype=np.int64)
    lib().cugo_ref_step(_p(rows), _p(actions), ctypes.c_int64(n), _p(reward), _p(done), _p(nagari),
                        _p(status), _p(committed), _p(ev), ctypes.c_int(threads or default_threads()))
    out = (rows, reward, done.astype(bool), nagari.astype(bool), status, committed.astype(bool))
    return out + (ev,) if events else out


def start(rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.zeros((rows.shape[0], START_WORDS), dtype=np.int64)
    lib().cugo_ref_start(_p(rows), ctypes.c_int64(rows.shape[0]), _p(out))
    return out


def hands(rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.zeros((rows.shape[0], 2), dtype=np.int64)
    lib().cugo_ref_hands(_p(rows), ctypes.c_int64(rows.shape[0]), _p(out))
    return out


def stock(rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.zeros(rows.shape[0], dtype=np.int64)
    lib().cugo_ref_stock(_p(rows), ctypes.c_int64(rows.shape[0]), _p(out))
    return out


def settle(row: np.ndarray) -> np.ndarray:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    out = np.zeros(10, dtype=np.int64)
    lib().cugo_ref_settle(_p(row), _p(out))
    return out


def rollout_random(game0: int, n: int, seed_base: int = 12345, max_decisions: int = 256,
                   stream: int = 0, threads: int | None = None):
    """Seeded random-legal games game0..game0+n-1 (oracle/driver.h)."""
    final_rows = np.zeros((n, STATE_BYTES), dtype=np.uint8)
    reward0 = np.zeros(n, dtype=np.int64)
    decisions = np.zeros(n, dtype=np.int32)
    events = np.zeros(n, dtype=np.int32)
    hashes = np.zeros(n, dtype=np.uint64)
    last_status = np.zeros(n, dtype=np.int16)
    lib().cugo_ref_rollout_random(
        ctypes.c_int64(game0), ctypes.c_int64(n), ctypes.c_int64(seed_base),
        ctypes.c_int(max_decisions), ctypes.c_uint32(stream), _p(final_rows), _p(reward0),
        _p(decisions), _p(events), _p(hashes), _p(last_status),
        ctypes.c_int(threads or default_threads()))
    return dict(final_rows=final_rows, reward0=reward0, decisions=decisions, events=events,
                hashes=hashes, last_status=last_status)


def branch_roots(n_roots: int, seed_base: int = 12345, threads: int | None = None) -> np.ndarray:
    rows = np.zeros((n_roots, STATE_BYTES), dtype=np.uint8)
    lib().cugo_ref_branch_roots(ctypes.c_int64(n_roots), ctypes.c_int64(seed_base), _p(rows),
                                ctypes.c_int(threads or default_threads()))
    return rows


def branch_actions(roots: np.ndarray, per_root: int, seed_base: int = 12345):
    roots = np.ascontiguousarray(roots, dtype=np.uint8)
    n = roots.shape[0] * per_root
    ids = np.zeros(n, dtype=np.int64)
    actions = np.zeros(n, dtype=np.int64)
    lib().cugo_ref_branch_actions(_p(roots), ctypes.c_int64(roots.shape[0]), ctypes.c_int64(per_root),
                                  ctypes.c_int64(seed_base), _p(ids), _p(actions))
    return ids, actions


def philox_word(game: int, decision: int, stream: int, seed: int) -> int:
    fn = lib().cugo_ref_philox_word
    fn.restype = ctypes.c_uint32
    fn.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64]
    return int(fn(game & (2**64 - 1), decision, stream, seed & (2**64 - 1)))
