"""ctypes binding of libpbgb200.so (the C ABI declared in include/pbgb200.h).

The library is built in-tree by ``ai-game-learning_b200/build.py``.  There is
no fallback: if the library is missing, or a tensor handed to it is not a
CUDA tensor, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpbgb200.so")

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


class NativeError(RuntimeError):
    """A libpbgb200 entry point returned a failure status."""


class Geometry(ctypes.Structure):
    _fields_ = [("players", _I32), ("stack_ticks", _I32), ("rank_count", _I32)]


class State(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "board", "combo", "button", "street", "to_act", "stacks", "committed", "committed_street",
        "status", "current_bet", "last_full_raise", "pending", "can_raise", "terminal")]


class History(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "actor", "street", "action", "amount", "pot_before", "call_amount", "current_bet",
        "min_raise_to", "max_raise_to", "mask")] + [("tokens", _I32), ("length", _P)]


class Leaf(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("board", "combo", "level", "baseline", "amount")]


class Policy(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("type_logits", "omega", "mu", "scale", "iota")] + [
        ("rows", _I32), ("mixtures", _I32)]


class TargetTables(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "work0", "work1", "trace", "cost", "delta", "head_v", "head_t", "head_c", "sigma_v", "sigma_t", "sigma_c",
        "action_p", "action_a", "work_cap", "head_cap", "width", "conversion")]


class TargetNodes(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "replica", "child_begin", "child_count", "destination_row", "input_type", "output_type", "owner_slot",
        "nominal_degree", "target_degree", "sigma_head_row", "sigma_target_row", "action_begin")]


class TargetChildren(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("source_row", "source_type", "path", "multiplier")]


class PolicyGrad(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("type_logits", "omega", "mu", "scale", "iota")]


G, S, Hs, L, Pol, PolG = Geometry, State, History, Leaf, Policy, PolicyGrad

SIGNATURES: dict[str, tuple] = {
    "pbg_last_error": (ctypes.c_char_p, []),
    "pbg_abi_version": (_I32, []),
    "pbg_rng_keys": (_I32, [_I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_child_path": (_I32, [_I64, _P, _P, _P, _P]),
    "pbg_logical_uniform": (_I32, [_I64, _P, _P, _P]),
    "pbg_logical_categorical": (_I32, [_I64, _I32, _P, _P, _P, _P, _P]),
    "pbg_initial_roots": (_I32, [G, _I64, _I64, _I64, _I64, _I64, _I64, _P, S, _P]),
    "pbg_legality": (_I32, [G, _I64, S, _P, _P]),
    "pbg_input_type": (_I32, [G, _I64, S, _P, _P]),
    "pbg_step_player": (_I32, [G, _I64, S, _P, _P]),
    "pbg_needs_chance": (_I32, [G, _I64, S, _P, _P]),
    "pbg_deal_next_street": (_I32, [G, _I64, S, _P, _P, _P]),
    "pbg_deal_next_street_keyed": (_I32, [G, _I64, S, _I64, _I64, _P, _P, _I64, _P, _P, _P, _P]),
    "pbg_append_player_history": (_I32, [G, _I64, S, _P, Hs, _P]),
    "pbg_append_chance_history": (_I32, [G, _I64, S, _P, Hs, _P]),
    "pbg_sampled_leaf": (_I32, [G, _I64, S, L, _P]),
    "pbg_combo_cards": (_I32, [G, _I64, _P, _P, _P]),
    "pbg_combo_class": (_I32, [G, _P, _P]),
    "pbg_direct_model_input": (_I32, [G, _I64, S, _I32, _P, Hs, _P, _I64, _P]),
    "pbg_evaluate_showdowns": (_I32, [_I32, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_hand_values": (_I32, [_I32, _I64, _P, _P, _P]),
    "pbg_rb_complete": (_I32, [_I32, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_rb_complete_max_samples": (_I32, [_I32, _I32]),
    "pbg_mlp_bias_relu": (_I32, [_I64, _I32, _P, _P, _P]),
    "pbg_mlp_heads": (_I32, [_I64, _I32, _I32, ctypes.c_float, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_mlp_heads_backward": (_I32, [_I64, _I32, _I32, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                      _I64, _P]),
    "pbg_mlp_bias_partials": (_I64, [_I64, _I32]),
    "pbg_mlp_relu_backward_bias": (_I32, [_I64, _I32, _P, _P, _P, _P, _I64, _P]),
    "pbg_gelu_backward": (_I32, [_I64, _I32, _P, _I64, _P, _I32, _I64, _P, _I64, _P]),
    "pbg_layernorm_backward_partials": (_I64, [_I64, _I32]),
    "pbg_layernorm_backward": (_I32, [_I64, _I32, _P, _I32, _I64, _P, ctypes.c_float, _P, _I32, _I64, _P, _I32, _I64, _P, _I64,
                                      _P]),
    "pbg_attention_backward": (_I32, [_I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_attention_bf16_lse": (_I32, [_I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_policy_probabilities": (_I32, [_I64, _I32, Pol, _P, _P, _P]),
    "pbg_policy_selected_log_pi": (_I32, [_I64, _I32, Pol, _P, _P, _P, _P]),
    "pbg_policy_entropy": (_I32, [_I64, _I32, Pol, _P, _P, _P]),
    "pbg_policy_sample_actor": (_I32, [_I64, _I32, Pol, _P, _P, _P, _P, _P, _P]),
    "pbg_learner_workspace_bytes": (_I64, [_I64, _I64, _I32]),
    "pbg_poker_learner_objective": (_I32, [_I64, _I64, _I32, _I32, _I32, Pol, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                           _P, _P, _P, _P, _P, _P, _P, PolG, _P, _P, _P, _P, _P, _I64, _P]),
    "pbg_policy_learner_forward": (_I32, [_I64, _I32, Pol, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_policy_learner_backward": (_I32, [_I64, _I32, Pol, _P, _P, _P, _P, _P, _P, PolG, _P]),
    "pbg_rollout_step": (_I32, [G, _I64, S, Hs, _P, _P, _P, _I64, _I64, Pol, _P, _P, _P, _P, L, _P]),
    "pbg_rollout_step_listed": (_I32, [G, _I64, S, Hs, _P, _P, _P, _I64, _I64, Pol, _P, _P, _P, _P, L, _P, _P]),
    "pbg_reach_update": (_I32, [G, _I64, S, Pol, _P, _P, _P, _P]),
    "pbg_ppo_partials_size": (_I64, [_I64, _I32]),
    "pbg_ppo_categorical_backward": (_I32, [_I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_ppo_categorical_backward_grid": (_I32, [_I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32,
                                                 _P]),
    "pbg_ppo_categorical_backward_noalloc": (_I32, [_I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_ppo_readout_partials_size": (_I64, [_I64, _I32, _I32]),
    "pbg_ppo_readout_backward": (_I32, [_I64, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _P, _P, _P, _P, _P]),
    "pbg_posterior_workspace_floats": (_I64, [G, _I64]),
    "pbg_posterior_sample_children": (_I32, [G, _I64, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _I64,
                                             _I32, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_alias_workspace_bytes": (_I64, [_I64]),
    "pbg_alias_table": (_I32, [_I64, _P, _P, _P, _P, _P]),
    "pbg_decision_log_mass": (_I32, [_I64, _P, _P, _P, _P, _P, _P]),
    "pbg_folded_query_count": (_I64, [_I32]),
    "pbg_folded_phi_queries": (_I32, [_I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_symmetric_eigh": (_I32, [_I64, _I32, _P, _P, _P, _I32, _P]),
    "pbg_layered_targets_workspace_words": (_I64, [_I32]),
    "pbg_layered_targets": (_I32, [_P, _I32, TargetNodes, TargetChildren, TargetTables, _I32, _I32, _I32, _I32,
                                   _I32, _I32, ctypes.c_float, _I32, _I32, _P, _P, _P]),
    "pbg_linear_bf16": (_I32, [_I64, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P]),
    "pbg_linear_gelu_backward": (_I32, [_I64, _I32, _I32, _P, _I64, _P, _P, _P, _P, _I64, _I64, _P, _I64, _P, _I64, _P,
                                        _P]),
    "pbg_linear_ex": (_I32, [_I64, _I32, _I32, _P, _I64, _P, _P, _P, _P, _I64, _I64, _P, _I64, _I32, _I32, _P, _P]),
    "pbg_layernorm_rows": (_I32, [_I64, _I32, _I64, _P, _I32, _I64, _I64, _P, _P, ctypes.c_float, _P, _I32, _I64,
                                  _I64, _P]),
    "pbg_scatter_rows_bf16": (_I32, [_I64, _I32, _I64, _P, _P, _I64, _I64, _P]),
    "pbg_incidence_combine_backward": (_I32, [_I64, _I32, _I64, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_incidence_combine": (_I32, [_I64, _I32, _I64, _I32, _P, _P, _P, _P, _I64, _I32, _I32, _P, _P, _I64, _I64,
                                     _I32, _I32, _P]),
    "pbg_attention_bf16": (_I32, [_I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "pbg_layernorm": (_I32, [_I64, _I32, _P, _I32, _P, _P, ctypes.c_float, _P, _I32, _I64, _P]),
    "pbg_nvls_signal_bytes": (_I64, []),
    "pbg_nvls_allreduce_sum_f32": (_I32, [_I64, _P, _P, _I64, _I32, _I32, _P, _P]),
    "pbg_nvls_allreduce_sum_f32_grid": (_I32, [_I64, _P, _P, _I64, _I32, _I32, _P, _I32, _P]),
    "pbg_adam_partials_size": (_I64, [_I64]),
    "pbg_adam_step": (_I32, [_I64, _P, _P, _P, _P, _P, _P, _I32, _P, _P, _P]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libpbgb200.so once; raise if it was not built."""

    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise NativeError(
                        f"{LIB_PATH} is missing: build it with `python ai-game-learning_b200/build.py`")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().pbg_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed ({rc}): {msg}")


_keep = threading.local()


def call(name: str, *args) -> None:
    """Invoke an entry point; tensors passed through ptr() stay alive until it returns.

    Without this, two temporaries built in one argument list (for example two
    ``torch.full_like`` columns) could share one caching-allocator block: the
    first is freed as soon as ptr() returns and the second reuses it.
    """

    try:
        check(getattr(lib(), name)(*args), name)
    finally:
        _keep.items = []


def ptr(t: torch.Tensor | None):
    """Device pointer of a contiguous CUDA tensor (None -> NULL), kept alive for call()."""

    if t is None:
        return None
    if not t.is_cuda:
        raise NativeError("libpbgb200 operates on CUDA tensors only")
    if not t.is_contiguous():
        raise NativeError("libpbgb200 requires contiguous tensors")
    items = getattr(_keep, "items", None)
    if items is None:
        items = _keep.items = []
    items.append(t)
    return ctypes.c_void_p(t.data_ptr())


def rows_ptr(t: torch.Tensor | None):
    """Device pointer of a CUDA matrix whose rows are contiguous (any row stride), kept alive for call()."""

    if t is None:
        return None
    if not t.is_cuda:
        raise NativeError("libpbgb200 operates on CUDA tensors only")
    if t.ndim != 2 or t.stride(1) != 1:
        raise NativeError("libpbgb200 requires a matrix with contiguous rows")
    items = getattr(_keep, "items", None)
    if items is None:
        items = _keep.items = []
    items.append(t)
    return ctypes.c_void_p(t.data_ptr())


def stream(device: torch.device | None = None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
