"""Composite poker policy on the device (pbg/games/poker/queued/policy.py).

``PokerPolicyOperator`` keeps the reference's entry points (probabilities,
selected_log_pi, policy_reductions, sample_actor, learner); each runs one
warp per policy row in libpbgb200.  ``learner`` and ``policy_reductions`` are
differentiable in the raw fields, as the reference's autograd path is.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from ._native import call, ptr, stream
from .learner import policy_learner
from .poker import CHECK_CALL, FOLD, RAISE_OFFSET, PokerLegality

_FIELDS = ("type_logits", "omega", "mu", "s", "iota")


class PokerPolicyError(ValueError):
    """Raw policy or public legality violates the canonical operation."""


@dataclass(frozen=True)
class ActorSample:
    action: Tensor
    selected_log_policy: Tensor


@dataclass(frozen=True)
class PolicyEvaluation:
    """pbg/core/learner.py:335-340."""

    selected_log_policy: Tensor
    entropy: Tensor
    reference_kl: Tensor


def policy_struct(raw: Mapping[str, Tensor]) -> tuple[N.Policy, tuple, int]:
    """Flatten raw fields to [rows, ...] fp32 and describe them for the ABI."""

    if set(raw) != set(_FIELDS):
        raise PokerPolicyError(f"raw policy fields must be exactly {sorted(_FIELDS)}")
    logits = raw["type_logits"]
    prefix = logits.shape[:-1]
    rows = 1 if len(prefix) == 1 else int(torch.tensor(prefix[1:]).prod())
    M = raw["omega"].shape[-1]
    keep = tuple(raw[n].float().contiguous() for n in _FIELDS)
    return N.Policy(*(ptr(t) for t in keep), rows, M), keep, rows


class PokerPolicyOperator:
    """policy.py:136-298."""

    def __init__(self, *, epsilon: float = 1.0e-12) -> None:
        if epsilon != 1.0e-12:
            raise ValueError("the device policy uses the reference epsilon 1e-12")
        self.epsilon = float(epsilon)

    @staticmethod
    def _mask(legality: PokerLegality) -> Tensor:
        E = legality.event_ids.shape[1]
        ids = torch.arange(E, dtype=legality.event_ids.dtype, device=legality.event_ids.device)
        if not torch.equal(legality.event_ids, ids[None].expand_as(legality.event_ids)):
            raise PokerPolicyError("device policy requires canonical event ids 0..E-1")
        return legality.mask.contiguous()

    def probabilities(self, raw: Mapping[str, Tensor], legality: PokerLegality) -> Tensor:
        pol, keep, rows = policy_struct(raw)
        mask = self._mask(legality)
        B, E = mask.shape
        out = torch.empty((B * rows, E), dtype=torch.float32, device=mask.device)
        call("pbg_policy_probabilities", B, E, pol, ptr(mask), ptr(out), stream(mask.device))
        return out.reshape(raw["type_logits"].shape[:-1] + (E,))

    def selected_log_pi(self, raw: Mapping[str, Tensor], legality: PokerLegality, action: Tensor) -> Tensor:
        pol, keep, rows = policy_struct(raw)
        mask = self._mask(legality)
        B, E = mask.shape
        if action.shape != (B,):
            raise PokerPolicyError("selected action must have shape [B]")
        out = torch.empty(B * rows, dtype=torch.float32, device=mask.device)
        call("pbg_policy_selected_log_pi", B, E, pol, ptr(mask), ptr(action.to(torch.int32).contiguous()), ptr(out),
             stream(mask.device))
        return out.reshape(raw["type_logits"].shape[:-1])

    def policy_reductions(self, raw: Mapping[str, Tensor], legality: PokerLegality,
                          reference_raw: Mapping[str, Tensor] | None = None) -> tuple[Tensor, Tensor]:
        """policy.py:235-244; differentiable in ``raw`` (pbg_policy_learner_forward / _backward)."""

        mask = self._mask(legality)
        action = torch.ones(mask.shape[0], dtype=torch.int32, device=mask.device)  # check/call: always legal
        _, entropy, kl = policy_learner(raw, mask, action, reference_raw)
        return entropy, kl

    def sample_actor(self, raw: Mapping[str, Tensor], legality: PokerLegality, actor_hand: Tensor,
                     logical_key: Tensor) -> ActorSample:
        if raw["type_logits"].ndim != 3 or actor_hand.shape != logical_key.shape \
                or actor_hand.shape != raw["type_logits"].shape[:1] or logical_key.dtype != torch.int64:
            raise PokerPolicyError("actor sampling requires policy [B,H,E] and aligned hands/keys")
        pol, keep, rows = policy_struct(raw)
        mask = self._mask(legality)
        B, E = mask.shape
        action = torch.empty(B, dtype=torch.int32, device=mask.device)
        selected = torch.empty(B, dtype=torch.float32, device=mask.device)
        call("pbg_policy_sample_actor", B, E, pol, ptr(mask), ptr(actor_hand.to(torch.int32).contiguous()),
             ptr(logical_key.contiguous()), ptr(action), ptr(selected), stream(mask.device))
        return ActorSample(action, selected)

    def learner(self, raw, legality, action, sampled_private_state, owner, reference_raw) -> PolicyEvaluation:
        """policy.py:284-298: selected log pi, entropy and reference KL in one pass per policy row,
        differentiable in ``raw`` through libpbgb200's vector-Jacobian product."""

        del sampled_private_state, owner
        mask = self._mask(legality)
        if action.shape != (mask.shape[0],):
            raise PokerPolicyError("selected action must have shape [B]")
        return PolicyEvaluation(*policy_learner(raw, mask, action, reference_raw))


__all__ = ["CHECK_CALL", "FOLD", "RAISE_OFFSET", "ActorSample", "PokerLegality", "PokerPolicyError",
           "PokerPolicyOperator", "PolicyEvaluation"]
