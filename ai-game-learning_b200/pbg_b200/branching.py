"""Branched learner sampling metadata: Walker alias tables and decision log mass.

``alias_table`` is pbg/core/learner.py:1519-1543 (``_alias_table``): scaled
weights ``n * softmax(log_weights)`` in float64, then the table.
``decision_log_path_mass`` is pbg/core/branching.py:113-141.  The operators
``AliasTableOperator.build_alias_table`` and ``BranchingOperator.decision_log_mass``
have the argument lists of the reference's two extension modules
(pbg/core/cuda_alias.py, pbg/core/cuda_branching.py).  Tables and masses are
identical to the reference kernels'; the work runs in ``pbg_alias_table`` and
``pbg_decision_log_mass``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ._native import NativeError, call, lib, ptr, stream


class LearnerError(RuntimeError):
    """pbg/core/learner.py LearnerError for the alias-table entry point."""


def _workspace(nbytes: int, device) -> Tensor:
    return torch.empty((nbytes + 15) // 16 * 2, dtype=torch.int64, device=device)


def build_alias_table(scaled: Tensor, probability: Tensor, alias: Tensor, small: Tensor | None = None,
                      large: Tensor | None = None) -> None:
    """alias_table.cu:47-89 ``build_alias_table``: fills probability / alias from scaled (consumed in place).

    ``small`` / ``large`` are accepted for the reference's signature; this build
    uses its own workspace instead of two index stacks.
    """

    n = scaled.numel()
    if not scaled.is_cuda or scaled.dtype != torch.float64 or scaled.ndim != 1 or n == 0 or not scaled.is_contiguous():
        raise NativeError("scaled weights must be contiguous CUDA FP64 [N]")
    if probability.dtype != torch.float64 or probability.shape != scaled.shape or not probability.is_contiguous():
        raise NativeError("probability must be contiguous CUDA FP64 [N]")
    if alias.dtype != torch.int32 or alias.shape != scaled.shape or not alias.is_contiguous():
        raise NativeError("alias must be contiguous CUDA int32 [N]")
    work = _workspace(int(lib().pbg_alias_workspace_bytes(n)), scaled.device)
    call("pbg_alias_table", n, ptr(scaled), ptr(probability), ptr(alias), ptr(work), stream(scaled.device))


def alias_table(log_weights: Tensor) -> tuple[Tensor, Tensor]:
    """learner.py:1519-1543: one deterministic Walker table in float64 -> (probability, alias)."""

    if log_weights.device.type != "cuda" or log_weights.ndim != 1 or log_weights.numel() == 0:
        raise LearnerError("alias log weights must be a nonempty CUDA vector")
    work = log_weights.detach().double()
    if not bool(torch.isfinite(work).all()):
        raise LearnerError("alias log weights must be finite")
    size = work.numel()
    scaled = (torch.exp(work - torch.logsumexp(work, 0)) * size).contiguous()
    probability = torch.empty_like(scaled)
    alias = torch.empty(size, dtype=torch.int32, device=work.device)
    build_alias_table(scaled, probability, alias)
    return probability, alias


def decision_log_mass(parent: Tensor, degree: Tensor, failure: Tensor) -> Tensor:
    """branching_metadata.cu:33-63 ``decision_log_mass``: log masses f32 [N]; failure int32 [1] gets 1 or 2."""

    if not parent.is_cuda or parent.dtype != torch.int32 or parent.ndim != 1 or not parent.is_contiguous():
        raise NativeError("parent must be contiguous CUDA int32 [N]")
    if degree.dtype != torch.int32 or degree.shape != parent.shape or not degree.is_contiguous():
        raise NativeError("degree must be contiguous CUDA int32 [N]")
    if failure.dtype != torch.int32 or failure.numel() != 1 or not failure.is_contiguous():
        raise NativeError("failure must be one contiguous CUDA int32")
    result = torch.empty(parent.shape, dtype=torch.float32, device=parent.device)
    work = _workspace(8, parent.device)
    call("pbg_decision_log_mass", parent.numel(), ptr(parent), ptr(degree), ptr(result), ptr(failure), ptr(work),
         stream(parent.device))
    return result


def decision_log_path_mass(parent: Tensor, executed_degree: Tensor, *, device: torch.device) -> Tensor:
    """branching.py:113-141: final log decision masses on CUDA from CPU topology columns."""

    if (parent.device.type != "cpu" or executed_degree.device.type != "cpu"
            or parent.dtype not in (torch.int32, torch.int64) or executed_degree.dtype not in (torch.int32, torch.int64)
            or parent.ndim != 1 or parent.shape != executed_degree.shape):
        raise ValueError("topology mass inputs must be aligned CPU integers")
    if torch.device(device).type != "cuda":
        raise ValueError("decision log mass requires a CUDA destination")
    failure = torch.zeros(1, dtype=torch.int32, device=device)
    result = decision_log_mass(parent.to(device=device, dtype=torch.int32),
                               executed_degree.to(device=device, dtype=torch.int32), failure)
    if int(failure.item()):
        raise ValueError("decision log mass encountered invalid topology")
    return result


class AliasTableOperator:
    """Module-like handle with the reference alias extension's entry point (cuda_alias.py:13)."""

    build_alias_table = staticmethod(build_alias_table)


class BranchingOperator:
    """Module-like handle with the reference branching extension's entry point (cuda_branching.py)."""

    decision_log_mass = staticmethod(decision_log_mass)


def alias_table_cuda() -> AliasTableOperator:
    return AliasTableOperator()


def branching_cuda() -> BranchingOperator:
    return BranchingOperator()


__all__ = ["AliasTableOperator", "BranchingOperator", "LearnerError", "alias_table", "alias_table_cuda",
           "branching_cuda", "build_alias_table", "decision_log_mass", "decision_log_path_mass"]
