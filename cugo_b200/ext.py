"""Drop-in for the reference's extension loader (python/cugo_torch50_ext.py:141-193).

``load_extension()`` returns an object with the reference module's 11 ops and 8
constants (python/csrc/torch50_ext.cpp:36-72): same names, argument order, output
shapes, dtypes, list return values and RuntimeError messages.  Each op checks its
tensors on the host, allocates its outputs with ``torch.empty`` on the states'
device and enqueues one kernel of libcugo_b200.so on the current CUDA stream — no
host synchronisation, so the ops can be captured in CUDA graphs.

There is no CPU path: without CUDA or without the native library the loader raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Any

import torch

from . import build as _build

_VP, _I64, _I32, _U32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_uint32

# name -> argument types after the leading pointers (all return int status)
_SIGNATURES: dict[str, list] = {
    "cugo_b200_create": [_VP, _VP, _I64, _VP, _VP],
    "cugo_b200_create_indexed": [_VP, _I64, _I64, _VP, _VP],
    "cugo_b200_running_init": [_VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _VP],
    "cugo_b200_observe": [_VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_observe_indexed": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_step": [_VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_step_indexed": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_step_events_indexed": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_branch_indexed": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_clone_indexed": [_VP, _I64, _VP, _I64, _VP, _VP],
    "cugo_b200_hands_indexed": [_VP, _I64, _VP, _I64, _VP, _VP],
    "cugo_b200_stock_indexed": [_VP, _I64, _VP, _I64, _VP, _VP],
    "cugo_b200_start": [_VP, _I64, _VP, _VP],
    "cugo_b200_rollout_random": [_I64, _I64, _I64, _I32, _U32, _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_selfplay_random_step": [_VP, _I64, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_branch_roots": [_I64, _I64, _VP, _VP],
    "cugo_b200_branch_actions": [_VP, _I64, _I64, _I64, _VP, _VP, _VP],
    "cugo_b200_sample_actions": [_VP, _I64, _VP, _I64, _VP, _VP, _I64, _I32, _VP, _VP, _VP],
    "cugo_b200_gemm_bf16": [_VP, _I64, _VP, _I64, _VP, _VP, _I64, _VP, _I64, _I32, _I32, _I32,
                            _I64, _I64, _I64, _VP, _VP],
    "cugo_b200_observe_indexed_bf16": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_gemm_bf16_ex": [_VP, _I64, _VP, _I64, _VP, _I32, _VP, _I64, _VP, _I64, _I32, _I32,
                               _I32, _I64, _I64, _I64, _VP, _VP],
    "cugo_b200_gemm_bf16_window": [_VP, _I64, _VP, _I64, _VP, _I32, _VP, _I64, _VP, _I64, _I32,
                                   _I32, _I32, _I64, _I64, _I64, _VP, _VP, _VP],
    "cugo_b200_gemm_bf16_pre": [_VP, _I64, _VP, _I64, _VP, _I32, _VP, _I64, _VP, _I64, _I32, _I64,
                                _I64, _I64, _VP, _VP],
    "cugo_b200_observe_query_bf16": [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _VP],
    "cugo_b200_observe_critic_bf16": [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP],
    "cugo_b200_redeal": [_VP, _I64, _VP, _I64, _I32, _VP],
    "cugo_b200_redeal_worlds": [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I32, _VP, _VP, _VP],
    "cugo_b200_encode_events": [_VP, _I64, _VP, _VP, _I64, _I32, _VP, _I32, _VP, _VP],
    "cugo_b200_games_attention": [_VP, _I64, _I64, _I32, _I32, _VP, ctypes.c_float, _VP, _I64,
                                  _VP],
    "cugo_b200_mlp_fused": [_VP, _I64, _I64, _I64, _I32, _VP, _VP, _I64, _I32, _VP, _I64, _VP,
                            _VP],
    "cugo_b200_mlp_fused_sample": [_VP, _I64, _I64, _I64, _I32, _VP, _VP, _I64, _I32, _VP, _VP,
                                   _VP, _VP, _I64, _I64, _I32, _VP, _VP, _VP, _I64, _VP, _VP,
                                   _VP],
    "cugo_b200_pack_legal": [_VP, _I64, _VP, _VP],
    "cugo_b200_observe_indexed_bf16_bits": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP,
                                            _VP],
    "cugo_b200_step_compact": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                               _VP, _VP],
    "cugo_b200_step_compact_grouped": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _VP, _VP,
                                       _VP, _VP, _VP],
    "cugo_b200_rowdot_bf16": [_VP, _I64, _VP, _VP, _I64, _I64, _VP, _I64, _VP],
    "cugo_b200_decode_attention": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _I64, _I32, _I32, _I32,
                                   _VP, _I64, _VP, _I64, ctypes.c_float, _VP, _I64, _VP, _VP],
    "cugo_b200_decode_attention_active": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _I64, _I32, _I32,
                                          _I32, _VP, _I64, _VP, _I64, ctypes.c_float, _VP, _I64,
                                          _VP, _VP, _VP],
    "cugo_b200_layernorm": [_VP, _I64, _VP, _VP, _I64, ctypes.c_float, _VP, _I64, _I64, _VP],
    "cugo_b200_event_embed": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _VP, _I64, _VP],
    "cugo_b200_start_embed": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _VP, _I64, _VP],
    "cugo_b200_record_transitions": [_VP, _I64, _VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP,
                                     _VP, _VP, _I32, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                                     _VP, _VP, _VP, _VP],
    "cugo_b200_wait_timeout_probe": [_I64, _VP, _VP, _VP],
    "cugo_b200_ppo_loss": [_VP, _I64, _VP, _VP, _VP, _VP, _VP, _I64, _VP, _I64, ctypes.c_float,
                           _VP, ctypes.c_float, _VP, _I64, _VP, _VP, _VP],
    "cugo_b200_colsum_bf16": [_VP, _I64, _VP, _I64, _I32, _VP, _I64, _I64, _I32, _VP, _VP, _I64,
                              _VP],
    "cugo_b200_scalar_head_backward": [_VP, _VP, _VP, _I64, _I32, _VP, _I64, _I64, _I32, _VP, _VP,
                                       _VP, _VP, _I64, _VP],
    "cugo_b200_wgrad_bf16": [_VP, _I64, _VP, _I64, _I64, _I64, _I64, _VP, _I64, _VP, _I64, _VP,
                             _VP],
    "cugo_b200_stock_planes_bf16": [_VP, _I64, _VP, _I64, _VP, _I64, _I32, _VP],
    "cugo_b200_wave_tail": [_I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                            _VP, _VP, _VP, _VP, _VP, _VP, _I32, _VP, _VP, _VP, _VP, _VP, _VP,
                            _VP, _VP, _VP, _I64, _VP],
}
_CONSTANTS = {
    "FEATURE_COUNT": "cugo_b200_feature_count",
    "ACTION_COUNT": "cugo_b200_action_count",
    "PRIMARY_ACTION_COUNT": "cugo_b200_primary_action_count",
    "CHOICE_ACTION_BEGIN": "cugo_b200_choice_action_begin",
    "EVENT_WORDS": "cugo_b200_event_words",
    "START_WORDS": "cugo_b200_start_words",
    "STATE_BYTES": "cugo_b200_state_bytes",
    "STATUS_OK": "cugo_b200_status_ok",
}
_EXTRA_CONSTANTS = {"EVENT_IN": "cugo_b200_event_inputs", "START_IN": "cugo_b200_start_inputs"}
_INT64_FUNCTIONS = {"cugo_b200_colsum_scratch_floats": [_I64, _I32],
                    "cugo_b200_wgrad_scratch_floats": [_I64, _I64, _I64],
                    "cugo_b200_running_init_scratch": [_I64]}
_ERRORS = {-1: "invalid argument", -2: "misaligned pointer", -3: "kernel launch failed"}

_LIB: ctypes.CDLL | None = None


def library_path() -> Path:
    return _build.LIB


def load_library(build_if_missing: bool = True) -> ctypes.CDLL:
    """dlopen libcugo_b200.so (building it first when it is missing)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = _build.LIB
    if not path.exists():
        if not build_if_missing:
            raise RuntimeError(f"cugo_b200 native library missing: {path}")
        _build.build()
    lib = ctypes.CDLL(str(path))
    for name, argtypes in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    for fn_name in [*_CONSTANTS.values(), *_EXTRA_CONSTANTS.values()]:
        getattr(lib, fn_name).restype = ctypes.c_int64
        getattr(lib, fn_name).argtypes = []
    for fn_name, argtypes in _INT64_FUNCTIONS.items():
        getattr(lib, fn_name).restype = ctypes.c_int64
        getattr(lib, fn_name).argtypes = argtypes
    lib.cugo_b200_abi_version.restype = ctypes.c_int
    _LIB = lib
    return lib


def _check(rc: int, op: str) -> None:
    if rc != 0:
        raise RuntimeError(f"cugo_b200 {op}: {_ERRORS.get(rc, f'error {rc}')}")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_cuda_1d(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.dim() != 1:
        raise RuntimeError(f"{name} must be one-dimensional")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} has the wrong dtype")


def _check_states(states: torch.Tensor, state_bytes: int) -> None:
    if not states.is_cuda:
        raise RuntimeError("states must be a CUDA tensor")
    if not states.is_contiguous():
        raise RuntimeError("states must be contiguous")
    if states.dtype != torch.uint8:
        raise RuntimeError("states must have dtype torch.uint8")
    if states.dim() != 2:
        raise RuntimeError("states must have shape [N, STATE_BYTES]")
    if states.size(1) != state_bytes:
        raise RuntimeError("states second dimension must equal STATE_BYTES")


def _same_device(a: torch.Tensor, b: torch.Tensor, an: str, bn: str) -> None:
    if a.device != b.device:
        raise RuntimeError(f"{an} and {bn} must be on the same CUDA device")


class CugoB200Extension:
    """The reference extension's op surface over libcugo_b200.so."""

    def __init__(self, lib: ctypes.CDLL) -> None:
        self._lib = lib
        for attr, fn_name in [*_CONSTANTS.items(), *_EXTRA_CONSTANTS.items()]:
            setattr(self, attr, int(getattr(lib, fn_name)()))

    # -- helpers ----------------------------------------------------------------
    @staticmethod
    def _stream(device: torch.device) -> int:
        return torch.cuda.current_stream(device).cuda_stream

    def _obs_outputs(self, m: int, device: torch.device) -> list[torch.Tensor]:
        return [
            torch.empty((m, self.FEATURE_COUNT), dtype=torch.float32, device=device),
            torch.empty((m, self.ACTION_COUNT), dtype=torch.bool, device=device),
            torch.empty((m,), dtype=torch.uint8, device=device),
            torch.empty((m,), dtype=torch.bool, device=device),
            torch.empty((m,), dtype=torch.int16, device=device),
        ]

    @staticmethod
    def _step_outputs(m: int, device: torch.device) -> list[torch.Tensor]:
        return [
            torch.empty((m,), dtype=torch.float32, device=device),
            torch.empty((m,), dtype=torch.bool, device=device),
            torch.empty((m,), dtype=torch.bool, device=device),
            torch.empty((m,), dtype=torch.int16, device=device),
            torch.empty((m,), dtype=torch.bool, device=device),
        ]

    def _states(self, states: torch.Tensor) -> None:
        _check_states(states, self.STATE_BYTES)

    # -- ops (python/csrc/torch50_ext.cpp:38-59) --------------------------------
    def create(self, seeds: torch.Tensor, first_players: torch.Tensor) -> torch.Tensor:
        _check_cuda_1d(seeds, torch.int64, "seeds")
        _check_cuda_1d(first_players, torch.int64, "first_players")
        if seeds.numel() != first_players.numel():
            raise RuntimeError("seeds and first_players must have the same length")
        _same_device(seeds, first_players, "seeds", "first_players")
        n = seeds.numel()
        with torch.cuda.device(seeds.device):
            states = torch.empty((n, self.STATE_BYTES), dtype=torch.uint8, device=seeds.device)
            _check(self._lib.cugo_b200_create(_ptr(seeds), _ptr(first_players), n, _ptr(states),
                                              self._stream(seeds.device)), "create")
        return states

    def create_indexed(self, index: torch.Tensor, seed_base: int) -> torch.Tensor:
        """create(index + seed_base, index & 1) in one kernel (see the C declaration)."""
        _check_cuda_1d(index, torch.int64, "index")
        n = index.numel()
        with torch.cuda.device(index.device):
            states = torch.empty((n, self.STATE_BYTES), dtype=torch.uint8, device=index.device)
            _check(self._lib.cugo_b200_create_indexed(_ptr(index), int(seed_base), n, _ptr(states),
                                                      self._stream(index.device)), "create_indexed")
        return states

    def running_init(self, states, ids, count, decision, reward0, nagari, bad,
                     scratch: torch.Tensor, spare_ids: torch.Tensor | None = None) -> None:
        """A fresh batch's running set (see the C declaration): ids int64 [>= n] gets the
        rows whose game the deal did not end (then i at position i), count int32 [1]
        their number, spare_ids (optional, int64 [>= n]) i at position i; decision int32,
        reward0 fp32, nagari bool [n] zeroed; bad int64 [1] zeroed; scratch int32
        [>= 2 * ceil(n / 32)]."""
        self._states(states)
        n = states.size(0)
        for t, dt, name in ((ids, torch.int64, "ids"), (count, torch.int32, "count"),
                            (decision, torch.int32, "decision"), (reward0, torch.float32, "reward0"),
                            (nagari, torch.bool, "nagari"), (bad, torch.int64, "bad"),
                            (scratch, torch.int32, "scratch")):
            if t.dtype != dt or not t.is_contiguous() or t.device != states.device:
                raise RuntimeError(f"running_init: {name} must be a contiguous {dt} tensor on the states' device")
        if ids.numel() < n or decision.numel() < n or reward0.numel() < n or nagari.numel() < n:
            raise RuntimeError("running_init: ids, decision, reward0 and nagari need n entries")
        if spare_ids is not None and (spare_ids.dtype != torch.int64 or spare_ids.numel() < n
                                      or not spare_ids.is_contiguous()
                                      or spare_ids.device != states.device):
            raise RuntimeError("running_init: spare_ids must be a contiguous int64 tensor of n entries")
        with torch.cuda.device(states.device):
            _check(self._lib.cugo_b200_running_init(
                _ptr(states), n, _ptr(ids), _ptr(spare_ids), _ptr(count), _ptr(decision),
                _ptr(reward0),
                _ptr(nagari), _ptr(bad), _ptr(scratch), scratch.numel(),
                self._stream(states.device)), "running_init")

    def observe(self, states: torch.Tensor) -> list[torch.Tensor]:
        self._states(states)
        n = states.size(0)
        with torch.cuda.device(states.device):
            out = self._obs_outputs(n, states.device)
            _check(self._lib.cugo_b200_observe(_ptr(states), n, *map(_ptr, out),
                                               self._stream(states.device)), "observe")
        return out

    def observe_indexed(self, states: torch.Tensor, env_ids: torch.Tensor) -> list[torch.Tensor]:
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            out = self._obs_outputs(m, states.device)
            _check(self._lib.cugo_b200_observe_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), m, *map(_ptr, out),
                self._stream(states.device)), "observe_indexed")
        return out

    def step(self, states: torch.Tensor, actions: torch.Tensor) -> list[torch.Tensor]:
        self._states(states)
        _check_cuda_1d(actions, torch.int64, "actions")
        if states.size(0) != actions.numel():
            raise RuntimeError("states and actions must have the same batch size")
        _same_device(states, actions, "states", "actions")
        n = states.size(0)
        with torch.cuda.device(states.device):
            out = self._step_outputs(n, states.device)
            _check(self._lib.cugo_b200_step(_ptr(states), n, _ptr(actions), *map(_ptr, out),
                                            self._stream(states.device)), "step")
        return out

    def _indexed_args(self, states, env_ids, actions) -> None:
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _check_cuda_1d(actions, torch.int64, "actions")
        if env_ids.numel() != actions.numel():
            raise RuntimeError("env_ids and actions must have the same length")
        _same_device(states, env_ids, "states", "env_ids")
        _same_device(states, actions, "states", "actions")

    def step_indexed(self, states, env_ids, actions) -> list[torch.Tensor]:
        self._indexed_args(states, env_ids, actions)
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            out = self._step_outputs(m, states.device)
            _check(self._lib.cugo_b200_step_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), _ptr(actions), m, *map(_ptr, out),
                self._stream(states.device)), "step_indexed")
        return out

    def step_events_indexed(self, states, env_ids, actions) -> list[torch.Tensor]:
        self._indexed_args(states, env_ids, actions)
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            out = self._step_outputs(m, states.device)
            events = torch.empty((m, self.EVENT_WORDS), dtype=torch.int64, device=states.device)
            _check(self._lib.cugo_b200_step_events_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), _ptr(actions), m, *map(_ptr, out),
                _ptr(events), self._stream(states.device)), "step_events_indexed")
        return out + [events]

    def clone_indexed(self, states, env_ids) -> torch.Tensor:
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            children = torch.empty((m, self.STATE_BYTES), dtype=torch.uint8, device=states.device)
            _check(self._lib.cugo_b200_clone_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), m, _ptr(children),
                self._stream(states.device)), "clone_indexed")
        return children

    def branch_indexed(self, states, env_ids, actions) -> list[torch.Tensor]:
        self._indexed_args(states, env_ids, actions)
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            children = torch.empty((m, self.STATE_BYTES), dtype=torch.uint8, device=states.device)
            out = self._step_outputs(m, states.device)
            _check(self._lib.cugo_b200_branch_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), _ptr(actions), m, _ptr(children),
                *map(_ptr, out), self._stream(states.device)), "branch_indexed")
        return [children] + out

    def hands_indexed(self, states, env_ids) -> torch.Tensor:
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            hands = torch.empty((m, 2), dtype=torch.int64, device=states.device)
            _check(self._lib.cugo_b200_hands_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), m, _ptr(hands),
                self._stream(states.device)), "hands_indexed")
        return hands

    def stock_indexed(self, states, env_ids) -> torch.Tensor:
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            stock = torch.empty((m,), dtype=torch.int64, device=states.device)
            _check(self._lib.cugo_b200_stock_indexed(
                _ptr(states), states.size(0), _ptr(env_ids), m, _ptr(stock),
                self._stream(states.device)), "stock_indexed")
        return stock

    def start(self, states) -> torch.Tensor:
        self._states(states)
        n = states.size(0)
        with torch.cuda.device(states.device):
            out = torch.empty((n, self.START_WORDS), dtype=torch.int64, device=states.device)
            _check(self._lib.cugo_b200_start(_ptr(states), n, _ptr(out),
                                             self._stream(states.device)), "start")
        return out

    # -- benchmark drivers (no counterpart in the reference extension) ----------
    def rollout_random(self, game0: int, n: int, seed_base: int = 12345, max_decisions: int = 256,
                       stream_id: int = 0, device: torch.device | str = "cuda") -> dict[str, Any]:
        device = torch.device(device)
        with torch.cuda.device(device):
            out = dict(
                final_rows=torch.empty((n, self.STATE_BYTES), dtype=torch.uint8, device=device),
                reward0=torch.empty((n,), dtype=torch.int64, device=device),
                decisions=torch.empty((n,), dtype=torch.int32, device=device),
                events=torch.empty((n,), dtype=torch.int32, device=device),
                hashes=torch.empty((n,), dtype=torch.int64, device=device),
                last_status=torch.empty((n,), dtype=torch.int16, device=device),
            )
            _check(self._lib.cugo_b200_rollout_random(
                game0, n, seed_base, max_decisions, stream_id, _ptr(out["final_rows"]),
                _ptr(out["reward0"]), _ptr(out["decisions"]), _ptr(out["events"]),
                _ptr(out["hashes"]), _ptr(out["last_status"]), self._stream(device)),
                "rollout_random")
        return out

    def selfplay_random_step(self, states, slot_game, slot_decision, slot_completed, slot_steps,
                             features, legal, seed_base: int = 12345,
                             actions: torch.Tensor | None = None) -> torch.Tensor:
        """One config-1 decision of every slot; returns the drawn actions."""
        n = states.size(0)
        with torch.cuda.device(states.device):
            if actions is None:
                actions = torch.empty((n,), dtype=torch.int64, device=states.device)
            _check(self._lib.cugo_b200_selfplay_random_step(
                _ptr(states), n, seed_base, _ptr(slot_game), _ptr(slot_decision),
                _ptr(slot_completed), _ptr(slot_steps), _ptr(features), _ptr(legal), _ptr(actions),
                self._stream(states.device)), "selfplay_random_step")
        return actions

    def branch_roots(self, n_roots: int, seed_base: int = 12345,
                     device: torch.device | str = "cuda") -> torch.Tensor:
        device = torch.device(device)
        with torch.cuda.device(device):
            roots = torch.empty((n_roots, self.STATE_BYTES), dtype=torch.uint8, device=device)
            _check(self._lib.cugo_b200_branch_roots(n_roots, seed_base, _ptr(roots),
                                                    self._stream(device)), "branch_roots")
        return roots

    def branch_actions(self, roots: torch.Tensor, per_root: int, seed_base: int = 12345):
        n = roots.size(0) * per_root
        with torch.cuda.device(roots.device):
            ids = torch.empty((n,), dtype=torch.int64, device=roots.device)
            actions = torch.empty((n,), dtype=torch.int64, device=roots.device)
            _check(self._lib.cugo_b200_branch_actions(
                _ptr(roots), roots.size(0), per_root, seed_base, _ptr(ids), _ptr(actions),
                self._stream(roots.device)), "branch_actions")
        return ids, actions


    def observe_indexed_bf16(self, states, env_ids) -> list[torch.Tensor]:
        """observe_indexed with bf16 features (the policy's input layer reads them)."""
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            out = self._obs_outputs(m, states.device)
            out[0] = torch.empty((m, self.FEATURE_COUNT), dtype=torch.bfloat16, device=states.device)
            _check(self._lib.cugo_b200_observe_indexed_bf16(
                _ptr(states), states.size(0), _ptr(env_ids), m, *map(_ptr, out),
                self._stream(states.device)), "observe_indexed_bf16")
        return out

    def observe_indexed_bf16_bits(self, states, env_ids,
                                  m_dev: torch.Tensor | None = None) -> list[torch.Tensor]:
        """observe_indexed_bf16 with the legal mask as int64 [m, 3] bit words (bit a of
        word a / 64) in place of the bool mask: [features, legal_bits, players, done,
        status]."""
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        dev = states.device
        with torch.cuda.device(dev):
            out = self._obs_outputs(m, dev)
            out[0] = torch.empty((m, self.FEATURE_COUNT), dtype=torch.bfloat16, device=dev)
            out[1] = torch.empty((m, 3), dtype=torch.int64, device=dev)
            _check(self._lib.cugo_b200_observe_indexed_bf16_bits(
                _ptr(states), states.size(0), _ptr(env_ids), m, *map(_ptr, out), _ptr(m_dev),
                self._stream(dev)), "observe_indexed_bf16_bits")
        return out

    def step_compact(self, states, env_ids, actions, decision, reward0, nagari, bad, next_ids,
                     next_count, scratch: torch.Tensor | None = None,
                     m_dev: torch.Tensor | None = None, grouped: bool = False) -> None:
        """step_indexed plus a self-play round's bookkeeping (see the C declaration):
        decision int32, reward0 fp32, nagari bool indexed by game id; bad int64 [1];
        next_ids int64 [>= m] and next_count int32 [1] receive the games still running,
        in order, or with `grouped` grouped by their next decision (primary plays,
        floor choices, prompts); scratch int32 [>= 2 (grouped: 6) * ceil(m / 32)]
        (allocated when not given)."""
        self._indexed_args(states, env_ids, actions)
        m = env_ids.numel()
        if next_ids.numel() < m or next_ids.dtype != torch.int64 or next_count.dtype != torch.int32:
            raise RuntimeError("step_compact: next_ids int64 [>= m], next_count int32 [1]")
        need = (6 if grouped else 2) * ((m + 31) // 32)
        if scratch is None:
            scratch = torch.empty(max(need, 1), dtype=torch.int32, device=states.device)
        if scratch.dtype != torch.int32 or scratch.numel() < need:
            raise RuntimeError(f"step_compact: scratch int32 [>= {need}]")
        fn = self._lib.cugo_b200_step_compact_grouped if grouped else self._lib.cugo_b200_step_compact
        with torch.cuda.device(states.device):
            _check(fn(
                _ptr(states), states.size(0), _ptr(env_ids), _ptr(actions), m, _ptr(decision),
                _ptr(reward0), _ptr(nagari), _ptr(bad), _ptr(next_ids), _ptr(next_count),
                _ptr(scratch), _ptr(m_dev), self._stream(states.device)), "step_compact")

    def record_transitions(self, states, active, m_dev, features, legal_bits, players, actions,
                           logp, learner, sizes, parity: int, store: dict, overflow) -> None:
        """Appends one collection round to a device-resident transition store (see the C
        declaration): round row i < min(active.numel(), *m_dev) goes to store row
        sizes[parity] + i; sizes[parity ^ 1] gets the new size.  store: bf16
        "features" [cap, 720], bool "legal" [cap, 179], int64 "actions", "opp_hand",
        "stock", "env_ids", "seat", fp32 "logp", bool "learner" [cap]."""
        self._states(states)
        m = active.numel()
        cap = store["actions"].numel()
        if features.dtype != torch.bfloat16 or features.stride(1) != 1 or features.shape[0] < m:
            raise RuntimeError("record_transitions: features bf16 [>= m, 720] with unit stride")
        if sizes.dtype != torch.int64 or sizes.numel() != 2:
            raise RuntimeError("record_transitions: sizes int64 [2]")
        with torch.cuda.device(states.device):
            _check(self._lib.cugo_b200_record_transitions(
                _ptr(states), states.size(0), _ptr(active), m, _ptr(m_dev), _ptr(features),
                features.stride(0), _ptr(legal_bits), _ptr(players), _ptr(actions), _ptr(logp),
                _ptr(learner), _ptr(sizes), parity, cap, _ptr(store["features"]),
                _ptr(store["legal"]), _ptr(store["actions"]), _ptr(store["logp"]),
                _ptr(store["opp_hand"]), _ptr(store["stock"]), _ptr(store["env_ids"]),
                _ptr(store["seat"]), _ptr(store["learner"]), _ptr(overflow),
                self._stream(states.device)), "record_transitions")

    def ppo_loss(self, logits: torch.Tensor, legal: torch.Tensor, actions: torch.Tensor,
                 logp_old: torch.Tensor, adv: torch.Tensor, value: torch.Tensor,
                 ret: torch.Tensor, clip: float, entropy_coef: torch.Tensor, value_coef: float,
                 dlogits: torch.Tensor, dvalue: torch.Tensor, stats: torch.Tensor) -> None:
        """The PPO minibatch losses and their gradients in one kernel (see the C
        declaration): logits fp32 [b, >=179] (rows may be padded), value fp32 [b] or
        [b, 1] (any row stride); writes dlogits bf16 [b, ldd >= 179] (pad columns 0),
        dvalue fp32 [b] and the five statistics' means into stats fp32 [5]."""
        b = logits.shape[0]
        if logits.dtype != torch.float32 or logits.stride(1) != 1 or logits.shape[1] < 179:
            raise RuntimeError("ppo_loss: logits fp32 [b, >= 179] with unit column stride")
        if dlogits.dtype != torch.bfloat16 or dlogits.stride(1) != 1 or dlogits.shape[0] != b:
            raise RuntimeError("ppo_loss: dlogits bf16 [b, >= 179]")
        if legal.dtype != torch.bool or not legal.is_contiguous() or legal.shape != (b, 179):
            raise RuntimeError("ppo_loss: legal bool [b, 179] contiguous")
        with torch.cuda.device(logits.device):
            _check(self._lib.cugo_b200_ppo_loss(
                _ptr(logits), logits.stride(0), _ptr(legal), _ptr(actions), _ptr(logp_old),
                _ptr(adv), _ptr(value), value.stride(0), _ptr(ret), b, float(clip),
                _ptr(entropy_coef), float(value_coef), _ptr(dlogits), dlogits.stride(0),
                _ptr(dvalue), _ptr(stats), self._stream(logits.device)), "ppo_loss")

    def _colsum_scratch(self, rows: int, n: int, device: torch.device) -> torch.Tensor:
        """The per-block partial sums' buffer, one per device, grown as needed (keep
        the sizes a CUDA graph replays within what it saw at capture)."""
        return self._scratch_floats(int(self._lib.cugo_b200_colsum_scratch_floats(rows, n)), device,
                                    "colsum")

    def _scratch_floats(self, need: int, device: torch.device, kind: str) -> torch.Tensor:
        """An fp32 scratch buffer per device, stream and kind of op (launches of one
        kind on one stream are ordered; two streams never share one), grown as
        needed."""
        cache = self.__dict__.setdefault("_scratch", {})
        key = (device, kind, torch.cuda.current_stream(device).cuda_stream)
        buf = cache.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(max(need, 1), dtype=torch.float32, device=device)
            cache[key] = buf
        return buf

    def colsum_bf16(self, x: torch.Tensor, out: torch.Tensor, z: torch.Tensor | None = None,
                    act: int = 0, dz: torch.Tensor | None = None) -> None:
        """out (fp32 [n]) = column sums of bf16 x [rows, n]; with z, of dz = x * act'(z),
        which is written to dz (bf16).  Deterministic (fixed summation order)."""
        rows, n = x.shape
        with torch.cuda.device(x.device):
            scratch = self._colsum_scratch(rows, n, x.device)
            _check(self._lib.cugo_b200_colsum_bf16(
                _ptr(x), x.stride(0), _ptr(z), z.stride(0) if z is not None else 0, act, _ptr(dz),
                dz.stride(0) if dz is not None else 0, rows, n, _ptr(out), _ptr(scratch),
                scratch.numel(), self._stream(x.device)), "colsum_bf16")

    def wgrad_bf16(self, dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor,
                   n_out: int | None = None, n_in: int | None = None) -> torch.Tensor:
        """out (fp32 [n_out, n_in]) = dy[:, :n_out]^T x[:, :n_in] over the rows on the
        tcgen05 tensor cores (bf16 operands, row-major; split over the rows, splits
        added in a fixed order)."""
        rows = dy.shape[0]
        n_out = dy.shape[1] if n_out is None else n_out
        n_in = x.shape[1] if n_in is None else n_in
        if dy.dtype != torch.bfloat16 or x.dtype != torch.bfloat16 or x.shape[0] != rows:
            raise RuntimeError("wgrad_bf16 expects bf16 dy [rows, n_out] and x [rows, n_in]")
        if dy.stride(1) != 1 or x.stride(1) != 1 or out.stride(1) != 1 or out.dtype != torch.float32:
            raise RuntimeError("wgrad_bf16 operands must be row-major, out fp32")
        with torch.cuda.device(dy.device):
            scratch = self._scratch_floats(
                int(self._lib.cugo_b200_wgrad_scratch_floats(rows, n_out, n_in)), dy.device, "wgrad")
            _check(self._lib.cugo_b200_wgrad_bf16(
                _ptr(dy), dy.stride(0), _ptr(x), x.stride(0), rows, n_out, n_in, _ptr(out),
                out.stride(0), _ptr(scratch), scratch.numel(), None, self._stream(dy.device)),
                "wgrad_bf16")
        return out

    def scalar_head_backward(self, dv: torch.Tensor, w: torch.Tensor, h: torch.Tensor, act: int,
                             dh: torch.Tensor, dh_sums: torch.Tensor, dw: torch.Tensor,
                             db: torch.Tensor) -> None:
        """Backward of a one-output head v = w . act(h) + b (see the C declaration)."""
        rows, n = h.shape
        with torch.cuda.device(h.device):
            scratch = self._colsum_scratch(rows, n, h.device)
            _check(self._lib.cugo_b200_scalar_head_backward(
                _ptr(dv), _ptr(w), _ptr(h), h.stride(0), act, _ptr(dh), dh.stride(0), rows, n,
                _ptr(dh_sums), _ptr(dw), _ptr(db), _ptr(scratch), scratch.numel(),
                self._stream(h.device)), "scalar_head_backward")

    def wait_timeout_probe(self, limit_ns: int, device: torch.device | str = "cuda"):
        """Runs the bounded mbarrier wait of the GEMM kernels on a barrier nothing
        arrives on: returns (error flag int32 [1], nanoseconds waited int64 [1])."""
        device = torch.device(device)
        with torch.cuda.device(device):
            error = torch.zeros(1, dtype=torch.int32, device=device)
            waited = torch.zeros(1, dtype=torch.int64, device=device)
            _check(self._lib.cugo_b200_wait_timeout_probe(limit_ns, _ptr(error), _ptr(waited),
                                                          self._stream(device)),
                   "wait_timeout_probe")
        return error, waited

    def stock_planes_bf16(self, states, env_ids, rows: torch.Tensor, first_column: int = 770) -> None:
        """Sets the one-hot planes of the next 8 stock draws (columns first_column ..
        + 400) in bf16 critic rows written by observe_critic_bf16 for the same ids."""
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        if rows.dtype != torch.bfloat16 or rows.stride(1) != 1 or rows.shape[0] != env_ids.numel():
            raise RuntimeError("stock_planes_bf16: rows bf16 [m, >= first_column + 400]")
        with torch.cuda.device(states.device):
            _check(self._lib.cugo_b200_stock_planes_bf16(
                _ptr(states), states.size(0), _ptr(env_ids), env_ids.numel(), _ptr(rows),
                rows.stride(0), first_column, self._stream(states.device)), "stock_planes_bf16")

    def wave_tail(self, obs_done, obs_status, players, actions, logp, step_out, wave: dict,
                  records: dict | None = None, learner: torch.Tensor | None = None) -> None:
        """The end of one sequence self-play decision step (see the C declaration).
        step_out: step_events_indexed's [reward0, done, nagari, status, committed,
        events]; wave: the wave's device state ("final_reward0", "final_nagari",
        "finished", "bad", "running", "events", "count", "cache_length", "decision",
        "step_index"); records: [max_steps, w] "actions", "seat", "count", "logp",
        "valid" (optional); learner: bool [w], whether the learner chose each action
        (optional)."""
        w = actions.numel()
        reward0, new_done, nagari, status, committed, events = step_out
        rec = records or {}
        max_steps = rec["actions"].shape[0] if records else 0
        with torch.cuda.device(actions.device):
            _check(self._lib.cugo_b200_wave_tail(
                w, _ptr(obs_done), _ptr(obs_status), _ptr(players), _ptr(actions), _ptr(logp),
                _ptr(reward0), _ptr(new_done), _ptr(nagari), _ptr(status), _ptr(committed),
                _ptr(events), _ptr(learner), _ptr(wave["final_reward0"]), _ptr(wave["final_nagari"]),
                _ptr(wave["finished"]), _ptr(wave["bad"]), _ptr(wave["running"]),
                _ptr(wave["events"]), wave["events"].shape[1], _ptr(wave["count"]),
                _ptr(wave["cache_length"]), _ptr(wave["decision"]), _ptr(wave["step_index"]),
                _ptr(rec.get("actions")), _ptr(rec.get("seat")), _ptr(rec.get("count")),
                _ptr(rec.get("logp")), _ptr(rec.get("valid")), max_steps,
                self._stream(actions.device)), "wave_tail")

    def pack_legal(self, legal: torch.Tensor) -> torch.Tensor:
        """bool [m, 179] legal masks as int64 [m, 3] bit words."""
        if legal.dtype != torch.bool or not legal.is_contiguous() or legal.dim() != 2 \
                or legal.shape[1] != self.ACTION_COUNT:
            raise RuntimeError("legal must be a contiguous bool [m, 179] tensor")
        m = legal.shape[0]
        bits = torch.empty((m, 3), dtype=torch.int64, device=legal.device)
        with torch.cuda.device(legal.device):
            _check(self._lib.cugo_b200_pack_legal(_ptr(legal), m, _ptr(bits),
                                                  self._stream(legal.device)), "pack_legal")
        return bits

    def observe_query_bf16(self, states, env_ids, query: torch.Tensor | None = None,
                           width: int = 904) -> list[torch.Tensor]:
        """observe_indexed writing the sequence policy's query input bf16 [m, width]:
        features in columns 0..719, legal as 0/1 in 720..898, zeros after."""
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        with torch.cuda.device(states.device):
            out = self._obs_outputs(m, states.device)
            if query is None:
                query = torch.empty((m, width), dtype=torch.bfloat16, device=states.device)
            if query.dtype != torch.bfloat16 or query.dim() != 2 or query.stride(1) != 1 or query.size(0) < m:
                raise RuntimeError("query must be a row-major bf16 [m, >=899] tensor")
            out[0] = query
            _check(self._lib.cugo_b200_observe_query_bf16(
                _ptr(states), states.size(0), _ptr(env_ids), m, _ptr(query), query.stride(0),
                *map(_ptr, out[1:]), self._stream(states.device)), "observe_query_bf16")
        return out

    def observe_critic_bf16(self, states, env_ids, width: int = 776) -> list[torch.Tensor]:
        """The oracle critic's input rows bf16 [m, width] (mover's features, the hand
        plane of the mover's opponent, zeros) plus players, done, status."""
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _same_device(states, env_ids, "states", "env_ids")
        m = env_ids.numel()
        dev = states.device
        with torch.cuda.device(dev):
            rows = torch.empty((m, width), dtype=torch.bfloat16, device=dev)
            players = torch.empty((m,), dtype=torch.uint8, device=dev)
            done = torch.empty((m,), dtype=torch.bool, device=dev)
            status = torch.empty((m,), dtype=torch.int16, device=dev)
            _check(self._lib.cugo_b200_observe_critic_bf16(
                _ptr(states), states.size(0), _ptr(env_ids), m, _ptr(rows), width, _ptr(players),
                _ptr(done), _ptr(status), self._stream(dev)), "observe_critic_bf16")
        return [rows, players, done, status]

    def redeal(self, rows: torch.Tensor, seats: torch.Tensor, seed: int, attempt: int = 0) -> None:
        """Redeals the rows in place for observer seats (the reference's _redeal)."""
        self._states(rows)
        _check_cuda_1d(seats, torch.int64, "seats")
        with torch.cuda.device(rows.device):
            _check(self._lib.cugo_b200_redeal(_ptr(rows), rows.size(0), _ptr(seats), seed, attempt,
                                              self._stream(rows.device)), "redeal")

    # -- policy layers -------------------------------------------------------------
    def linear(self, a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
               residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
               act: int = 0, act_after: int = 0, out_dtype: torch.dtype = torch.bfloat16,
               error: torch.Tensor | None = None,
               window: torch.Tensor | None = None) -> torch.Tensor:
        """out = act_after(act(a @ w.T + bias) + residual) on tcgen05 tensor cores.

        act codes: 0 none, 1 ReLU, 2 SiLU, 3 GELU (erf).  bias may be bf16 or fp32;
        the residual has the output's dtype (an fp32 stream may be updated in place,
        residual is out)."""
        m, k = a.shape
        n = w.shape[0]
        if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or w.shape[1] != k:
            raise RuntimeError("linear expects bf16 a [m, k] and w [n, k]")
        if a.stride(1) != 1 or w.stride(1) != 1:
            raise RuntimeError("linear operands must be row-major")
        if out is None:
            out = torch.empty((m, n), dtype=out_dtype, device=a.device)
        if residual is not None and residual.dtype != out.dtype:
            raise RuntimeError("linear residual must have the output's dtype")
        if bias is not None and bias.dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError("linear bias must be bf16 or fp32")
        args = (_ptr(a), a.stride(0), _ptr(w), w.stride(0), _ptr(bias),
                int(bias is not None and bias.dtype == torch.float32), _ptr(residual),
                residual.stride(0) if residual is not None else 0, _ptr(out), out.stride(0),
                int(out.dtype == torch.float32), act, act_after, m, n, k)
        with torch.cuda.device(a.device):
            if window is None:
                _check(self._lib.cugo_b200_gemm_bf16_ex(*args, _ptr(error), self._stream(a.device)),
                       "gemm_bf16")
            else:
                if window.dtype != torch.int32 or window.numel() < 2 or not window.is_cuda:
                    raise RuntimeError("linear window must be a CUDA int32 tensor {first row, rows}")
                _check(self._lib.cugo_b200_gemm_bf16_window(*args, _ptr(window), _ptr(error),
                                                            self._stream(a.device)), "gemm_bf16_window")
        return out

    def linear_pre(self, a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, act: int,
                   pre: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """out = act(a @ w.T + bias) and pre = a @ w.T + bias (both bf16) in one GEMM
        launch: a training forward's layer that keeps its pre-activation."""
        m, k = a.shape
        n = w.shape[0]
        if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or w.shape[1] != k:
            raise RuntimeError("linear_pre expects bf16 a [m, k] and w [n, k]")
        if pre.dtype != torch.bfloat16 or pre.shape != (m, n) or pre.stride(1) != 1:
            raise RuntimeError("linear_pre needs a row-major bf16 pre [m, n]")
        if out is None:
            out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
        if bias is not None and bias.dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError("linear bias must be bf16 or fp32")
        with torch.cuda.device(a.device):
            _check(self._lib.cugo_b200_gemm_bf16_pre(
                _ptr(a), a.stride(0), _ptr(w), w.stride(0), _ptr(bias),
                int(bias is not None and bias.dtype == torch.float32), _ptr(out), out.stride(0),
                _ptr(pre), pre.stride(0), act, m, n, k, None, self._stream(a.device)), "gemm_bf16_pre")
        return out

    def redeal_worlds(self, states, env_ids, seats, worlds: int, seed: int = 0, tries: int = 8,
                      with_attempts: bool = False):
        """[worlds * R, 248] redealt copies of states[env_ids] keeping each observer's
        view (one launch); with_attempts also returns the int8 attempt kept (-1: none)."""
        self._states(states)
        _check_cuda_1d(env_ids, torch.int64, "env_ids")
        _check_cuda_1d(seats, torch.int64, "seats")
        _same_device(states, env_ids, "states", "env_ids")
        r = env_ids.numel()
        if seats.numel() != r:
            raise RuntimeError("redeal_worlds: one seat per env id")
        dev = states.device
        with torch.cuda.device(dev):
            out = torch.empty((worlds * r, self.STATE_BYTES), dtype=torch.uint8, device=dev)
            acc = torch.empty((worlds * r,), dtype=torch.int8, device=dev) if with_attempts else None
            _check(self._lib.cugo_b200_redeal_worlds(
                _ptr(states), states.size(0), _ptr(env_ids), r, _ptr(seats), worlds, seed, tries,
                _ptr(out), _ptr(acc), self._stream(dev)), "redeal_worlds")
        return (out, acc) if with_attempts else out

    def encode_events(self, events: torch.Tensor, count: torch.Tensor, seats: torch.Tensor,
                      length: int, dtype: torch.dtype = torch.float32):
        """encode_events (python/cugo_seq50.py:91-109): tokens [B, length, 414] of dtype
        (fp32 or bf16) and the validity mask [B, length]."""
        if events.dtype != torch.int64 or events.dim() != 3 or events.size(2) != self.EVENT_WORDS \
                or not events.is_contiguous():
            raise RuntimeError("events must be a contiguous int64 [B, max_events, 9] tensor")
        if dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("encode_events writes fp32 or bf16 tokens")
        _check_cuda_1d(count, torch.int64, "count")
        _check_cuda_1d(seats, torch.int64, "seats")
        b = events.size(0)
        dev = events.device
        with torch.cuda.device(dev):
            tokens = torch.empty((b, length, self.EVENT_IN), dtype=dtype, device=dev)
            valid = torch.empty((b, length), dtype=torch.bool, device=dev)
            _check(self._lib.cugo_b200_encode_events(
                _ptr(events), events.size(1), _ptr(count), _ptr(seats), b, length, _ptr(tokens),
                int(dtype == torch.bfloat16), _ptr(valid), self._stream(dev)), "encode_events")
        return tokens, valid

    def games_attention(self, qkv: torch.Tensor, n_seq: int, length: int, queries: int,
                        seen: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Attention of SeqNet.forward_games over the three token blocks of qkv."""
        if qkv.dtype != torch.bfloat16 or qkv.dim() != 2 or qkv.stride(1) != 1:
            raise RuntimeError("qkv must be row-major bf16 [rows, 768]")
        rows = n_seq * (1 + length + queries)
        if qkv.size(0) != rows:
            raise RuntimeError("games_attention: qkv must hold n_seq * (1 + length + queries) rows")
        if out is None:
            out = torch.empty((rows, 256), dtype=torch.bfloat16, device=qkv.device)
        with torch.cuda.device(qkv.device):
            _check(self._lib.cugo_b200_games_attention(
                _ptr(qkv), qkv.stride(0), n_seq, length, queries, _ptr(seen), 32 ** -0.5, _ptr(out),
                out.stride(0), self._stream(qkv.device)), "games_attention")
        return out

    def mlp_fused(self, x: torch.Tensor, weights: list[torch.Tensor],
                  biases: list[torch.Tensor | None], act: int, out: torch.Tensor | None = None,
                  error: torch.Tensor | None = None) -> torch.Tensor:
        """The whole hidden-512 residual MLP in one kernel: fp32 [m, n_out] outputs.
        weights bf16 contiguous [out, in] (input layer, fc1/fc2 per block, head),
        biases fp32 (or None)."""
        m, k_in = x.shape
        if x.dtype != torch.bfloat16 or x.stride(1) != 1:
            raise RuntimeError("mlp_fused expects row-major bf16 x")
        if any(w.dtype != torch.bfloat16 or not w.is_contiguous() for w in weights):
            raise RuntimeError("mlp_fused expects contiguous bf16 weights")
        if weights[0].shape[0] != 512 or weights[0].shape[1] != k_in:
            raise RuntimeError("mlp_fused expects hidden 512 and an input weight [512, k_in]")
        if any(b is not None and (b.dtype != torch.float32 or not b.is_contiguous()) for b in biases):
            raise RuntimeError("mlp_fused expects contiguous fp32 biases")
        n_out = weights[-1].shape[0]
        if out is None:
            out = torch.empty((m, (n_out + 3) // 4 * 4), dtype=torch.float32,
                              device=x.device)[:, :n_out]
        wp = (ctypes.c_void_p * len(weights))(*[w.data_ptr() for w in weights])
        bp = (ctypes.c_void_p * len(biases))(*[b.data_ptr() if b is not None else None for b in biases])
        with torch.cuda.device(x.device):
            _check(self._lib.cugo_b200_mlp_fused(
                _ptr(x), x.stride(0), m, k_in, (len(weights) - 2) // 2, wp, bp, n_out, act,
                _ptr(out), out.stride(0), _ptr(error), self._stream(x.device)), "mlp_fused")
        return out

    def mlp_fused_sample(self, x: torch.Tensor, weights: list[torch.Tensor],
                         biases: list[torch.Tensor | None], act: int, legal: torch.Tensor,
                         game: torch.Tensor, decision: torch.Tensor, seed_base: int = 12345,
                         greedy: bool = False, want_logits: bool = False,
                         m_dev: torch.Tensor | None = None, rows: torch.Tensor | None = None):
        """The hidden-512 MLP and the masked Gumbel-max sampling of its first 179
        outputs in one kernel: (actions int64 [m], logp fp32 [m], logits or None).
        legal: bool [m, 179], or the int64 [m, 3] bit words of observe_indexed_bf16_bits.
        rows (optional int64 [m]): row r's game and decision are game[rows[r]] and
        decision[rows[r]] (an entry outside the arrays samples nothing: -1, log p 0)."""
        m, k_in = x.shape
        if x.dtype != torch.bfloat16 or x.stride(1) != 1:
            raise RuntimeError("mlp_fused_sample expects row-major bf16 x")
        if any(w.dtype != torch.bfloat16 or not w.is_contiguous() for w in weights):
            raise RuntimeError("mlp_fused_sample expects contiguous bf16 weights")
        if weights[0].shape[0] != 512 or weights[0].shape[1] != k_in:
            raise RuntimeError("mlp_fused_sample expects hidden 512 and an input weight [512, k_in]")
        if legal.dtype == torch.bool:
            legal = self.pack_legal(legal)
        if legal.dtype != torch.int64 or not legal.is_contiguous() or legal.shape != (m, 3):
            raise RuntimeError("legal must be a bool [m, 179] mask or its int64 [m, 3] bit words")
        _check_cuda_1d(game, torch.int64, "game")
        _check_cuda_1d(decision, torch.int32, "decision")
        if rows is not None:
            _check_cuda_1d(rows, torch.int64, "rows")
            if rows.numel() != m or game.numel() != decision.numel():
                raise RuntimeError("rows needs one entry per row and game, decision of one length")
        elif game.numel() != m or decision.numel() != m:
            raise RuntimeError("game and decision need one entry per row")
        n_out = weights[-1].shape[0]
        dev = x.device
        actions = torch.empty((m,), dtype=torch.int64, device=dev)
        logp = torch.empty((m,), dtype=torch.float32, device=dev)
        out = (torch.empty((m, (n_out + 3) // 4 * 4), dtype=torch.float32, device=dev)[:, :n_out]
               if want_logits else None)
        wp = (ctypes.c_void_p * len(weights))(*[w.data_ptr() for w in weights])
        bp = (ctypes.c_void_p * len(biases))(*[b.data_ptr() if b is not None else None for b in biases])
        with torch.cuda.device(dev):
            _check(self._lib.cugo_b200_mlp_fused_sample(
                _ptr(x), x.stride(0), m, k_in, (len(weights) - 2) // 2, wp, bp, n_out, act,
                _ptr(legal), _ptr(game), _ptr(decision), _ptr(rows), game.numel(), seed_base,
                int(greedy), _ptr(actions),
                _ptr(logp), _ptr(out), out.stride(0) if out is not None else 0, _ptr(m_dev), None,
                self._stream(dev)), "mlp_fused_sample")
        return actions, logp, out

    def rowdot(self, a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """out[r] = a[r] . w + bias: a one-output layer, bf16 a [m, k], fp32 w [k]."""
        m, k = a.shape
        if a.dtype != torch.bfloat16 or a.stride(1) != 1 or w.dtype != torch.float32:
            raise RuntimeError("rowdot expects row-major bf16 a and fp32 w")
        if not w.is_contiguous() or w.numel() != k:
            raise RuntimeError("rowdot: w must be a contiguous [k] vector")
        if out is None:
            out = torch.empty((m,), dtype=torch.float32, device=a.device)
        with torch.cuda.device(a.device):
            _check(self._lib.cugo_b200_rowdot_bf16(
                _ptr(a), a.stride(0), _ptr(w), _ptr(bias), m, k, _ptr(out),
                out.stride(0), self._stream(a.device)), "rowdot_bf16")
        return out

    # -- sequence policy decode ----------------------------------------------------
    def decode_attention(self, q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                         pos: torch.Tensor, rows: torch.Tensor | None = None,
                         k_new: torch.Tensor | None = None, v_new: torch.Tensor | None = None,
                         pos_clamp: int = -1, out: torch.Tensor | None = None,
                         error: torch.Tensor | None = None,
                         active: torch.Tensor | None = None) -> torch.Tensor:
        """decode_attention (python/cugo_seq_attention50.py:43-57) on the native kernel.

        q [n, heads, dh] bf16 (dh = 32, rows of q may be strided), keys/values
        [rows, heads, slots, dh] bf16 contiguous, pos/rows int64 -> out [n, heads, dh].
        k_new/v_new ([n, heads, dh]) are first written to slot pos of each row.
        pos_clamp >= 0: pos is the per-row length array, position = min(pos[row], clamp).
        active (bool [n]): only those queries attend and append; the others get zeros."""
        n, heads, dh = q.shape
        if q.dtype != torch.bfloat16 or keys.dtype != torch.bfloat16 or values.dtype != torch.bfloat16:
            raise RuntimeError("decode_attention expects bf16 q, keys and values")
        if q.stride(2) != 1 or q.stride(1) != dh or not keys.is_contiguous() or not values.is_contiguous():
            raise RuntimeError("decode_attention: q heads must be packed, keys/values contiguous")
        if keys.shape != values.shape or keys.dim() != 4 or keys.shape[1] != heads or keys.shape[3] != dh:
            raise RuntimeError("decode_attention: keys/values must be [rows, heads, slots, dh]")
        if (k_new is None) != (v_new is None):
            raise RuntimeError("decode_attention: pass both k_new and v_new or neither")
        ldn = 0
        if k_new is not None:
            if k_new.stride() != v_new.stride() or k_new.stride(2) != 1 or k_new.stride(1) != dh:
                raise RuntimeError("decode_attention: k_new/v_new must match q's layout")
            ldn = k_new.stride(0)
        if out is None:
            out = torch.empty((n, heads, dh), dtype=torch.bfloat16, device=q.device)
        with torch.cuda.device(q.device):
            if active is None:
                _check(self._lib.cugo_b200_decode_attention(
                    _ptr(q), q.stride(0), _ptr(k_new), _ptr(v_new), ldn, _ptr(keys), _ptr(values),
                    keys.shape[0], heads, keys.shape[2], dh, _ptr(pos), pos_clamp, _ptr(rows), n,
                    float(dh ** -0.5), _ptr(out), out.stride(0), _ptr(error),
                    self._stream(q.device)), "decode_attention")
            else:
                _check_cuda_1d(active, torch.bool, "active")
                if active.numel() != n:
                    raise RuntimeError("decode_attention: active must have one entry per query")
                _check(self._lib.cugo_b200_decode_attention_active(
                    _ptr(q), q.stride(0), _ptr(k_new), _ptr(v_new), ldn, _ptr(keys), _ptr(values),
                    keys.shape[0], heads, keys.shape[2], dh, _ptr(pos), pos_clamp, _ptr(rows), n,
                    float(dh ** -0.5), _ptr(out), out.stride(0), _ptr(active), _ptr(error),
                    self._stream(q.device)), "decode_attention")
        return out

    def layernorm(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                  eps: float = 1e-5, out: torch.Tensor | None = None) -> torch.Tensor:
        """nn.LayerNorm of fp32 rows into bf16 rows."""
        n, d = x.shape
        if x.dtype != torch.float32 or x.stride(1) != 1:
            raise RuntimeError("layernorm expects row-major fp32 x")
        if out is None:
            out = torch.empty((n, d), dtype=torch.bfloat16, device=x.device)
        with torch.cuda.device(x.device):
            _check(self._lib.cugo_b200_layernorm(
                _ptr(x), x.stride(0), _ptr(weight), _ptr(bias), d, float(eps), _ptr(out),
                out.stride(0), n, self._stream(x.device)), "layernorm")
        return out

    def event_embed(self, events: torch.Tensor, seats: torch.Tensor, index: torch.Tensor | None,
                    weight_t: torch.Tensor, bias: torch.Tensor, position: torch.Tensor,
                    token_type: torch.Tensor, n: int | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """Event tokens fp32 [n, d]; row i reads events[i % len(events)] and seats[i]."""
        if events.dtype != torch.int64 or not events.is_contiguous() or events.dim() != 2 \
                or events.size(1) != self.EVENT_WORDS:
            raise RuntimeError("events must be a contiguous int64 [n, 9] tensor")
        n = seats.numel() if n is None else n
        d = weight_t.shape[1]
        if out is None:
            out = torch.empty((n, d), dtype=torch.float32, device=events.device)
        with torch.cuda.device(events.device):
            _check(self._lib.cugo_b200_event_embed(
                _ptr(events), events.size(0), _ptr(seats), _ptr(index), n, _ptr(weight_t),
                _ptr(bias), _ptr(position), _ptr(token_type), d, _ptr(out), out.stride(0),
                self._stream(events.device)), "event_embed")
        return out

    def start_embed(self, start: torch.Tensor, seats: torch.Tensor, weight_t: torch.Tensor,
                    bias: torch.Tensor, position0: torch.Tensor, token_type: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """Opening tokens fp32 [n, d]; row i reads start[i % len(start)] and seats[i]."""
        if start.dtype != torch.int64 or not start.is_contiguous() or start.dim() != 2 \
                or start.size(1) != self.START_WORDS:
            raise RuntimeError("start must be a contiguous int64 [n, 8] tensor")
        n = seats.numel()
        d = weight_t.shape[1]
        if out is None:
            out = torch.empty((n, d), dtype=torch.float32, device=start.device)
        with torch.cuda.device(start.device):
            _check(self._lib.cugo_b200_start_embed(
                _ptr(start), start.size(0), _ptr(seats), n, _ptr(weight_t), _ptr(bias),
                _ptr(position0), _ptr(token_type), d, _ptr(out), out.stride(0),
                self._stream(start.device)), "start_embed")
        return out

    # -- policy sampling ---------------------------------------------------------
    def sample_actions(self, logits: torch.Tensor, legal: torch.Tensor, game: torch.Tensor,
                       decision: torch.Tensor, seed_base: int = 12345, greedy: bool = False):
        """Masked Gumbel-max (or greedy) actions and their log-probabilities."""
        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise RuntimeError("logits must be a row-major float32 [N, >=179] tensor")
        m = logits.size(0)
        with torch.cuda.device(logits.device):
            actions = torch.empty((m,), dtype=torch.int64, device=logits.device)
            logp = torch.empty((m,), dtype=torch.float32, device=logits.device)
            _check(self._lib.cugo_b200_sample_actions(
                _ptr(logits), logits.stride(0), _ptr(legal), m, _ptr(game), _ptr(decision),
                seed_base, int(greedy), _ptr(actions), _ptr(logp), self._stream(logits.device)),
                "sample_actions")
        return actions, logp


_EXT: CugoB200Extension | None = None


def load_extension(*, verbose: bool = False) -> CugoB200Extension:
    """Same contract as the reference's load_extension(): CUDA is required."""
    if not torch.cuda.is_available():
        raise RuntimeError("PyTorch CUDA is not available")
    global _EXT
    if _EXT is None:
        _EXT = CugoB200Extension(load_library())
    return _EXT
