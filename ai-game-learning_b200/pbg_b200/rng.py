"""Counter-based logical RNG on the device (pbg/core/rollout.py:73-267).

Same signatures and semantics as the reference: keys depend only on the
logical address (seed, iteration, purpose, root, path, draw, lane, retry
epoch), never on batching, order or stream.
"""

from __future__ import annotations

from enum import IntEnum

import torch
from torch import Tensor

from ._native import call, ptr, stream


class DrawPurpose(IntEnum):
    """rollout.py:73-86: closed counter namespaces."""

    PRIVATE = 1
    ROUND = 2
    POSTERIOR = 3
    ACTION = 4
    CHANCE = 5
    COMPLETION = 6
    LEARNER = 7
    ROLE_SELECTION = 8


LOGICAL_RNG_VERSION = "counter_hash_v4"


def _i64(reference: Tensor, value) -> Tensor:
    if isinstance(value, Tensor):
        return value.to(dtype=torch.int64, device=reference.device)
    return torch.full_like(reference, int(value), dtype=torch.int64)


def logical_rng_keys(*, seed: int, iteration: int, root: Tensor, path: Tensor, draw, purpose,
                     lane=0, retry_epoch=0, active: Tensor | None = None) -> Tensor:
    """rollout.py:122-181."""

    if root.device != path.device:
        raise ValueError("root and path addresses must share a device")
    if int(purpose) <= 0:
        raise ValueError("draw purpose must be a positive namespace identifier")
    root, path = torch.broadcast_tensors(root.to(torch.int64), path.to(torch.int64))
    cols = torch.broadcast_tensors(root, path, _i64(root, draw), _i64(root, lane), _i64(root, retry_epoch))
    flat = [c.contiguous().reshape(-1) for c in cols]
    out = torch.empty_like(flat[0])
    act = None
    if active is not None:
        if active.device != root.device:
            raise ValueError("active RNG mask must share the key device")
        act = torch.broadcast_to(active.to(torch.bool), cols[0].shape).contiguous().reshape(-1).view(torch.uint8)
    call("pbg_rng_keys", int(seed), int(iteration), int(purpose), flat[0].numel(), *map(ptr, flat), ptr(act),
         ptr(out), stream(root.device))
    return out.reshape(cols[0].shape)


def child_path_keys(parent_path: Tensor, child_ordinal) -> Tensor:
    """rollout.py:184-202."""

    ordinal = _i64(parent_path, child_ordinal)
    parent, ordinal = torch.broadcast_tensors(parent_path.to(torch.int64), ordinal)
    if not parent.is_cuda and not bool((ordinal > 0).all()):
        raise ValueError("child ordinals must be positive")
    p = parent.contiguous().reshape(-1)
    o = ordinal.contiguous().reshape(-1)
    out = torch.empty_like(p)
    call("pbg_child_path", p.numel(), ptr(p), ptr(o), ptr(out), stream(p.device))
    return out.reshape(parent.shape)


def logical_uniform(keys: Tensor, *, dtype: torch.dtype = torch.float32, active: Tensor | None = None) -> Tensor:
    """rollout.py:205-234."""

    if keys.dtype != torch.int64:
        raise ValueError("logical RNG keys must be int64")
    k = keys.contiguous().reshape(-1)
    out = torch.empty(k.shape, dtype=torch.float32, device=k.device)
    call("pbg_logical_uniform", k.numel(), ptr(k), ptr(out), stream(k.device))
    out = out.reshape(keys.shape).to(dtype)
    if active is not None:
        out = torch.where(torch.broadcast_to(active.to(torch.bool), out.shape), out, torch.zeros_like(out))
    return out


def logical_categorical(probability: Tensor, keys: Tensor, *, mass: Tensor | None = None,
                        active: Tensor | None = None) -> Tensor:
    """rollout.py:237-267."""

    if probability.ndim != 2 or keys.shape != probability.shape[:1]:
        raise ValueError("probability must be [B,E] and keys [B]")
    if probability.device != keys.device or keys.dtype != torch.int64:
        raise ValueError("probability and int64 keys must share a device")
    p = probability.float().contiguous()
    m = None if mass is None else mass.float().contiguous()
    out = torch.empty(keys.shape, dtype=torch.int64, device=keys.device)
    call("pbg_logical_categorical", p.shape[0], p.shape[1], ptr(p), ptr(keys.contiguous()), ptr(m), ptr(out),
         stream(p.device))
    if active is not None:
        out = torch.where(active, out, torch.full_like(out, -1))
    return out
