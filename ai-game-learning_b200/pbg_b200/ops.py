"""libpbgb200 entry points registered as torch custom operators.

A call into the shared library is opaque to ``torch.compile``; registered as a
custom operator with a shape function (``register_fake``) it becomes one node
of a traced graph, so a host program that compiles and CUDA-graph-captures its
learner step (pbg's tensor programs, pbg/core/execution_program.py:63-140)
keeps doing so with these kernels inside.  Registered here:

* ``pbg_b200::legality`` -- the legal events of B public states (the state
  machine's ``legality``, hooks.py:464-510);
* ``pbg_b200::poker_learner_objective`` -- the fused poker learner objective
  (learner.py:1824-2159 + the backward of the lane totals), whose autograd
  formula scales the gradients it computed in the forward by the upstream
  gradient of each lane's total.

Each operator allocates its outputs (and the objective its statistics
workspace) with torch, so inside a CUDA graph they come from the graph's pool.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _native as N
from ._native import call, ptr, stream

_FIELDS = ("type_logits", "omega", "mu", "s", "iota")
# launches per operator (counted in the implementations, which a tracer never enters: a captured
# graph's replays do not count)
CALLS = {"legality": 0, "poker_learner_objective": 0}


@torch.library.custom_op("pbg_b200::legality", mutates_args=())
def legality(board: Tensor, combo: Tensor, button: Tensor, street: Tensor, to_act: Tensor, stacks: Tensor,
             committed: Tensor, committed_street: Tensor, status: Tensor, current_bet: Tensor,
             last_full_raise: Tensor, pending: Tensor, can_raise: Tensor, terminal: Tensor, players: int,
             stack_ticks: int, rank_count: int) -> Tensor:
    CALLS["legality"] += 1
    rows = board.shape[0]
    mask = torch.empty((rows, stack_ticks + 2), dtype=torch.bool, device=board.device)
    cols = (board, combo, button, street, to_act, stacks, committed, committed_street, status, current_bet,
            last_full_raise, pending, can_raise, terminal)
    state = N.State(*(ptr(t.contiguous()) for t in cols))
    call("pbg_legality", N.Geometry(players, stack_ticks, rank_count), rows, state, ptr(mask), stream(board.device))
    return mask


@legality.register_fake
def _(board, combo, button, street, to_act, stacks, committed, committed_street, status, current_bet,
      last_full_raise, pending, can_raise, terminal, players, stack_ticks, rank_count):
    return board.new_empty((board.shape[0], stack_ticks + 2), dtype=torch.bool)


@torch.library.custom_op("pbg_b200::poker_learner_objective", mutates_args=())
def poker_learner_objective(type_logits: Tensor, omega: Tensor, mu: Tensor, s: Tensor, iota: Tensor,
                            ref_type_logits: Optional[Tensor], ref_omega: Optional[Tensor], ref_mu: Optional[Tensor],
                            ref_s: Optional[Tensor], ref_iota: Optional[Tensor], mask: Tensor,
                            action_ptr: Optional[Tensor], action: Tensor, old_log_policy: Tensor, advantage: Tensor,
                            posterior: Optional[Tensor], value: Tensor, old_value: Tensor, value_target: Tensor,
                            trace_pred: Optional[Tensor], cost_pred: Optional[Tensor], trace_target: Optional[Tensor],
                            cost_target: Optional[Tensor], controls: Tensor, lane_weight: Tensor
                            ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(result [lanes,10], d type_logits, d omega, d mu, d s, d iota, d value, d trace, d cost); the
    gradients are of sum_l lane_weight_l * total_l (d trace / d cost are empty without public heads)."""

    CALLS["poker_learner_objective"] += 1
    S, W, M = omega.shape
    E = mask.shape[1]
    A = action.shape[0]
    lanes = controls.shape[0]
    f32 = lambda t: None if t is None else t.detach().float().contiguous()  # noqa: E731
    raw = [f32(t) for t in (type_logits, omega, mu, s, iota)]
    pol = N.Policy(*(ptr(t) for t in raw), W, M)
    ref = None
    if ref_type_logits is not None:
        ref_cols = [f32(t) for t in (ref_type_logits, ref_omega, ref_mu, ref_s, ref_iota)]
        ref = N.Policy(*(ptr(t) for t in ref_cols), W, M)
    grads = [torch.empty_like(t) for t in raw]
    gstruct = N.PolicyGrad(*(ptr(t) for t in grads))
    dev = mask.device
    d_value = torch.empty((S, W), dtype=torch.float32, device=dev)
    heads = trace_pred is not None
    d_trace = torch.empty(S if heads else 0, dtype=torch.float32, device=dev)
    d_cost = torch.empty(S if heads else 0, dtype=torch.float32, device=dev)
    result = torch.empty((lanes, 10), dtype=torch.float32, device=dev)
    need = int(N.lib().pbg_learner_workspace_bytes(S, A, lanes))
    if need < 0:
        raise ValueError("learner lanes must lie in [1, 16]")
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    m = mask.contiguous().view(torch.uint8) if mask.dtype == torch.bool else mask.contiguous()
    call("pbg_poker_learner_objective", S, A, E, W, lanes, pol, None if ref is None else ctypes.byref(ref), ptr(m),
         ptr(None if action_ptr is None else action_ptr.to(torch.int64).contiguous()),
         ptr(action.to(torch.int32).contiguous()), ptr(f32(old_log_policy)), ptr(f32(advantage)), ptr(f32(posterior)),
         ptr(f32(value)), ptr(f32(old_value)), ptr(f32(value_target)), ptr(f32(trace_pred)), ptr(f32(cost_pred)),
         ptr(f32(trace_target)), ptr(f32(cost_target)), ptr(f32(controls)), ptr(f32(lane_weight)), gstruct,
         ptr(d_value), ptr(d_trace if heads else None), ptr(d_cost if heads else None), ptr(result), ptr(ws),
         ws.numel(), stream(dev))
    return (result, *grads, d_value, d_trace, d_cost)


@poker_learner_objective.register_fake
def _(type_logits, omega, mu, s, iota, ref_type_logits, ref_omega, ref_mu, ref_s, ref_iota, mask, action_ptr,
      action, old_log_policy, advantage, posterior, value, old_value, value_target, trace_pred, cost_pred,
      trace_target, cost_target, controls, lane_weight):
    S, W = omega.shape[:2]
    f = torch.float32
    heads = trace_pred is not None
    return (controls.new_empty((controls.shape[0], 10), dtype=f),
            *(t.new_empty(t.shape, dtype=f) for t in (type_logits, omega, mu, s, iota)),
            value.new_empty((S, W), dtype=f), value.new_empty((S if heads else 0,), dtype=f),
            value.new_empty((S if heads else 0,), dtype=f))


def _setup(ctx, inputs, output):
    lanes = inputs[23].shape[0]
    S = inputs[10].shape[0]
    ctx.lanes, ctx.S = lanes, S
    ctx.heads = inputs[19] is not None
    ctx.shapes = [inputs[i].shape for i in (0, 1, 2, 3, 4, 16)]
    ctx.dtypes = [inputs[i].dtype for i in (0, 1, 2, 3, 4, 16, 19, 20)] if ctx.heads else \
        [inputs[i].dtype for i in (0, 1, 2, 3, 4, 16)]
    ctx.save_for_backward(*output[1:])


def _backward(ctx, g_result, *unused):
    saved = ctx.saved_tensors
    per_sigma = g_result[:, 0].float().repeat_interleave(ctx.S // ctx.lanes)  # [S]

    def scaled(g, dtype):
        return (g * per_sigma.reshape((ctx.S,) + (1,) * (g.dim() - 1))).to(dtype)

    raw_grads = [scaled(saved[i], ctx.dtypes[i]).reshape(ctx.shapes[i]) for i in range(5)]
    d_value = scaled(saved[5], ctx.dtypes[5]).reshape(ctx.shapes[5])
    d_trace = scaled(saved[6], ctx.dtypes[6]) if ctx.heads else None
    d_cost = scaled(saved[7], ctx.dtypes[7]) if ctx.heads else None
    return (*raw_grads, None, None, None, None, None, None, None, None, None, None, None, d_value, None, None,
            d_trace, d_cost, None, None, None, None)


poker_learner_objective.register_autograd(_backward, setup_context=_setup)


__all__ = ["legality", "poker_learner_objective"]
