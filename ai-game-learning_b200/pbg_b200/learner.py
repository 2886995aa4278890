"""The poker learner objective and its gradient on the device (pbg/core/learner.py:1824-2159).

``PokerLearnerObjective`` runs ``LearnerOperation.forward_loss`` for one
physical batch with the poker policy operation
(pbg/games/poker/queued/policy.py:284-298 through hooks.py:2200-2246) and the
backward of ``(total * objective_weight * loss_scale).sum()``
(pbg/core/training.py:403) as ONE launch of libpbgb200's
``pbg_poker_learner_objective``: composite policy forward, PPO / Rao-Blackwell
rows, value, entropy, reference KL, trace and cost heads, lane means, and the
gradient of every raw policy field, the value and the public heads.

``poker_learner_loss`` runs the same launch as the ``pbg_b200::poker_learner_objective``
operator (pbg_b200.ops), whose autograd formula scales the per-lane gradients
it computed by the upstream gradient of each lane's total, so the model's
weight gradients follow from the usual ``.backward()`` -- eagerly or inside a
torch.compile'd, CUDA-graph-captured step.  ``policy_learner`` is the differentiable
``PokerPolicyOperator.learner`` (selected log pi, entropy, reference KL).

Batch layout (the reference's names):

* ``raw`` fields ``type_logits [S,W,3]``, ``omega/mu/s [S,W,M]``,
  ``iota [S,W]``: the sampled private row (W = 1) or every private hand
  (W = H, Rao-Blackwell);
* ``mask [S,E]`` legal events of each sigma row;
* ``action_ptr [S+1]`` ragged action spans of branched batches (None: unit);
* ``action [A]``, ``old_log_policy / advantage_target / posterior [A,W]``;
* ``value / old_value / value_target [S,W]``;
* ``controls [lanes,10]`` (``LearnerOperation.controls`` order) and
  ``lane_weight [lanes]`` (objective weight x loss scale).
"""

from __future__ import annotations

import ctypes
from collections.abc import Mapping
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from ._native import call, ptr, stream

_FIELDS = ("type_logits", "omega", "mu", "s", "iota")
RESULT_FIELDS = ("total", "policy", "value", "entropy", "reference_kl", "approximate_kl", "clip_fraction",
                 "negative_advantage_cap_fraction", "negative_advantage_log_ratio_max",
                 "negative_advantage_influence_max")


class LearnerError(ValueError):
    """A learner batch violates the loss contract (learner.py: LearnerError)."""


@dataclass(frozen=True)
class LossResult:
    """learner.py:1739-1749, one entry per lane."""

    total: Tensor
    policy: Tensor
    value: Tensor
    entropy: Tensor
    reference_kl: Tensor
    approximate_kl: Tensor
    clip_fraction: Tensor
    negative_advantage_cap_fraction: Tensor
    negative_advantage_log_ratio_max: Tensor
    negative_advantage_influence_max: Tensor

    @classmethod
    def from_rows(cls, result: Tensor) -> "LossResult":
        return cls(*(result[:, i] for i in range(len(RESULT_FIELDS))))


def _raw_struct(raw: Mapping[str, Tensor], S: int, W: int, keep: list) -> N.Policy:
    if set(raw) != set(_FIELDS):
        raise LearnerError(f"raw policy fields must be exactly {sorted(_FIELDS)}")
    M = raw["omega"].shape[-1]
    shapes = {"type_logits": (S, W, 3), "omega": (S, W, M), "mu": (S, W, M), "s": (S, W, M), "iota": (S, W)}
    cols = []
    for name in _FIELDS:
        t = raw[name]
        if tuple(t.shape) != shapes[name]:
            raise LearnerError(f"raw field {name} has shape {tuple(t.shape)}, expected {shapes[name]}")
        t = t.detach().float().contiguous()
        keep.append(t)
        cols.append(ptr(t))
    return N.Policy(*cols, W, M)


def _mask_u8(mask: Tensor) -> Tensor:
    return mask.contiguous().view(torch.uint8) if mask.dtype == torch.bool else mask.contiguous()


class PokerLearnerObjective:
    """Owns the workspace of the fused objective (grown on demand, zeroed once)."""

    def __init__(self, device) -> None:
        self.device = torch.device(device)
        self.workspace = torch.zeros(0, dtype=torch.uint8, device=self.device)

    def _workspace(self, S: int, A: int, lanes: int) -> Tensor:
        need = int(N.lib().pbg_learner_workspace_bytes(S, A, lanes))
        if need < 0:
            raise LearnerError("learner lanes must lie in [1, 16]")
        if self.workspace.numel() < need:
            self.workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self.workspace

    def __call__(self, raw: Mapping[str, Tensor], mask: Tensor, action: Tensor, old_log_policy: Tensor,
                 advantage: Tensor, value: Tensor, old_value: Tensor, value_target: Tensor, controls: Tensor,
                 lane_weight: Tensor, *, posterior: Tensor | None = None, action_ptr: Tensor | None = None,
                 reference_raw: Mapping[str, Tensor] | None = None, trace_pred: Tensor | None = None,
                 cost_pred: Tensor | None = None, trace_target: Tensor | None = None,
                 cost_target: Tensor | None = None) -> tuple[LossResult, dict]:
        """One launch; returns (LossResult per lane, gradients keyed by input name)."""

        S, E = mask.shape
        if raw["type_logits"].ndim != 3:
            raise LearnerError("raw fields must be [S, W, ...]")
        W = raw["type_logits"].shape[1]
        A = action.shape[0]
        lanes = controls.shape[0]
        if controls.shape != (lanes, 10) or lane_weight.shape != (lanes,):
            raise LearnerError("loss controls must be [K,10] with one lane weight per lane")
        if action_ptr is None and A != S:
            raise LearnerError("ragged learner batches need action_ptr")
        for name, t, shape in (("old_log_policy", old_log_policy, (A, W)), ("advantage_target", advantage, (A, W)),
                               ("value", value, (S, W)), ("old_value", old_value, (S, W)),
                               ("value_target", value_target, (S, W))):
            if t.numel() != shape[0] * shape[1] or t.shape[0] != shape[0]:
                raise LearnerError(f"{name} must be {shape}")
        if W > 1 and posterior is None:
            raise LearnerError("Rao-Blackwell rows need the posterior")
        keep: list = []
        pol = _raw_struct(raw, S, W, keep)
        ref = None if reference_raw is None else _raw_struct(reference_raw, S, W, keep)

        def f32(t):
            return None if t is None else t.detach().float().contiguous()

        old, adv, post = f32(old_log_policy), f32(advantage), f32(posterior)
        v, ov, tg = f32(value), f32(old_value), f32(value_target)
        tp, cp, tt, ct = f32(trace_pred), f32(cost_pred), f32(trace_target), f32(cost_target)
        ctl, lw = f32(controls), f32(lane_weight)
        act = action.to(torch.int32).contiguous()
        aptr = None if action_ptr is None else action_ptr.to(torch.int64).contiguous()
        dev = mask.device
        grads = {name: torch.empty_like(keep[i]) for i, name in enumerate(_FIELDS)}
        gstruct = N.PolicyGrad(*(ptr(grads[n]) for n in _FIELDS))
        d_value = torch.empty((S, W), dtype=torch.float32, device=dev)
        heads = trace_pred is not None
        d_trace = torch.empty(S, dtype=torch.float32, device=dev) if heads else None
        d_cost = torch.empty(S, dtype=torch.float32, device=dev) if heads else None
        result = torch.empty((lanes, 10), dtype=torch.float32, device=dev)
        ws = self._workspace(S, A, lanes)
        call("pbg_poker_learner_objective", S, A, E, W, lanes, pol, None if ref is None else ctypes.byref(ref),
             ptr(_mask_u8(mask)), ptr(aptr), ptr(act), ptr(old), ptr(adv), ptr(post), ptr(v), ptr(ov), ptr(tg),
             ptr(tp), ptr(cp), ptr(tt), ptr(ct), ptr(ctl), ptr(lw), gstruct, ptr(d_value), ptr(d_trace), ptr(d_cost),
             ptr(result), ptr(ws), ws.numel(), stream(dev))
        out = dict(grads)
        out["value"] = d_value
        if heads:
            out["trace_pred"] = d_trace
            out["cost_pred"] = d_cost
        return LossResult.from_rows(result), out


def poker_learner_loss(objective: "PokerLearnerObjective | None", raw: Mapping[str, Tensor], value: Tensor, *,
                       mask: Tensor, action: Tensor, old_log_policy: Tensor, advantage_target: Tensor,
                       old_value: Tensor, value_target: Tensor, controls: Tensor, posterior: Tensor | None = None,
                       action_ptr: Tensor | None = None, reference_raw: Mapping[str, Tensor] | None = None,
                       trace_pred: Tensor | None = None, cost_pred: Tensor | None = None,
                       trace_target: Tensor | None = None, cost_target: Tensor | None = None) -> LossResult:
    """Differentiable ``forward_loss``: a LossResult whose ``total`` [lanes] backpropagates into ``raw``,
    ``value`` and the public heads (the other fields are statistics without gradient).

    Runs the ``pbg_b200::poker_learner_objective`` operator, which torch.compile can trace and a CUDA
    graph can capture; ``objective`` is accepted for symmetry with the non-autograd entry and unused."""

    from .ops import poker_learner_objective as objective_op

    del objective
    S, E = mask.shape
    if raw["type_logits"].ndim != 3:
        raise LearnerError("raw fields must be [S, W, ...]")
    W = raw["type_logits"].shape[1]
    if action_ptr is None and action.shape[0] != S:
        raise LearnerError("ragged learner batches need action_ptr")
    if W > 1 and posterior is None:
        raise LearnerError("Rao-Blackwell rows need the posterior")
    ref = [None] * 5 if reference_raw is None else [reference_raw[n] for n in _FIELDS]
    lanes = controls.shape[0]
    ones = torch.ones(lanes, dtype=torch.float32, device=controls.device)
    out = objective_op(*(raw[n] for n in _FIELDS), *ref, mask, action_ptr, action, old_log_policy, advantage_target,
                       posterior, value, old_value, value_target, trace_pred, cost_pred, trace_target, cost_target,
                       controls.float(), ones)
    result = out[0]
    return LossResult(result[:, 0], *(result[:, i].detach() for i in range(1, len(RESULT_FIELDS))))


class _PolicyLearnerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, mask, action, reference_raw, *fields):
        raw = dict(zip(_FIELDS, fields, strict=True))
        B, rows = raw["iota"].shape
        E = mask.shape[1]
        keep: list = []
        pol = _raw_struct(raw, B, rows, keep)
        ref = None if reference_raw is None else _raw_struct(reference_raw, B, rows, keep)
        dev = mask.device
        sel = torch.empty((B, rows), dtype=torch.float32, device=dev)
        ent = torch.empty_like(sel)
        kl = torch.empty_like(sel)
        act = action.to(torch.int32).contiguous()
        call("pbg_policy_learner_forward", B, E, pol, None if ref is None else ctypes.byref(ref), ptr(mask), ptr(act),
             ptr(sel), ptr(ent), ptr(kl), stream(dev))
        ctx.save_for_backward(mask, act, *keep)
        ctx.has_ref = ref is not None
        ctx.dims = (B, rows, E)
        if reference_raw is None:
            ctx.mark_non_differentiable(kl)
        return sel, ent, kl

    @staticmethod
    def backward(ctx, g_sel, g_ent, g_kl):
        mask, act, *keep = ctx.saved_tensors
        B, rows, E = ctx.dims
        raw_keep, ref_keep = keep[:5], keep[5:]
        M = raw_keep[1].shape[-1]
        pol = N.Policy(*(ptr(t) for t in raw_keep), rows, M)
        ref = N.Policy(*(ptr(t) for t in ref_keep), rows, M) if ctx.has_ref else None
        grads = [torch.empty_like(t) for t in raw_keep]
        gstruct = N.PolicyGrad(*(ptr(t) for t in grads))

        def flat(t):
            return None if t is None else t.float().contiguous().reshape(-1)

        gk = flat(g_kl) if ctx.has_ref else None
        call("pbg_policy_learner_backward", B, E, pol, None if ref is None else ctypes.byref(ref), ptr(mask),
             ptr(act), ptr(flat(g_sel)), ptr(flat(g_ent)), ptr(gk), gstruct, stream(mask.device))
        return (None, None, None, *grads)


def policy_learner(raw: Mapping[str, Tensor], mask: Tensor, action: Tensor,
                   reference_raw: Mapping[str, Tensor] | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """Differentiable selected log pi, entropy and reference KL (policy.py:284-298).

    ``raw`` [B, rows, ...] (or [B, ...] for one row per decision), ``mask``
    [B, E] bool / uint8, ``action`` [B].  Gradients flow to ``raw`` only.
    """

    m = _mask_u8(mask)
    single = raw["type_logits"].ndim == 2
    fields = [raw[n].unsqueeze(1) if single else raw[n] for n in _FIELDS]
    ref = None
    if reference_raw is not None:
        ref = {n: reference_raw[n].unsqueeze(1) if single else reference_raw[n] for n in _FIELDS}
    sel, ent, kl = _PolicyLearnerFn.apply(m, action, ref, *fields)
    if single:
        return sel[:, 0], ent[:, 0], kl[:, 0]
    return sel, ent, kl


__all__ = ["LearnerError", "LossResult", "PokerLearnerObjective", "RESULT_FIELDS", "poker_learner_loss",
           "policy_learner"]
