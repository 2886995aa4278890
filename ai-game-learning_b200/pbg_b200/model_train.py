"""Backward of the policy/value network on this build's kernels: the learner step at cfg2.

The reference's learner step (pbg/core/training.py:336-424) runs the model
forward on the learner rows, ``LearnerOperation.forward_loss``, then
``(total * objective_weight * loss_scale).sum().backward()`` through torch
autograd and the optimizer.  Here the forward is the same tensor-core network
(``PreflopModel`` / ``PostflopModel`` in training mode) with each native step
wrapped in an autograd function whose backward is written for it:

- ``_LinearFn`` (``pbg_linear_ex``: ``act(x W^T * s + b + r)``): for a GELU
  map the same tcgen05 kernel recomputes the pre-activation and writes
  dY = dy * GELU'(pre) from its epilogue (``pbg_linear_gelu_backward``), then
  dX = dY W and dW = dY^T X as bf16 library GEMMs with fp32 accumulation (fp32
  dW), the bias and residual gradients as sums;
- ``_LayerNormFn`` (``pbg_layernorm``): ``pbg_layernorm_backward``;
- ``_AttentionFn`` (``pbg_attention_bf16_lse``, which also keeps each row's
  log-sum-exp): ``pbg_attention_backward``, one fused pass that recomputes the
  scores tile by tile on the tensor cores and gives dQ, dK, dV and the gradient
  of each head's score scale (so of the temperature parameter theta);
- ``_IncidenceCombineFn`` (``pbg_incidence_combine``, the incidence residual's
  seat sums): ``pbg_incidence_combine_backward``.

The key bias and mask of the attention and the row mass of the incidence map
come from the learner rows' ranges, not from parameters, and get no gradient.

``ModelLearnerStep`` is the whole step over one learner batch of each family:
the forward with every parameter a leaf view of one flat fp32 master whose
gradient views share one flat buffer, the fused poker objective
(``PokerLearnerObjective``), the backward, and ``FlatAdam``.
"""

from __future__ import annotations

import ctypes
import math

import torch
from torch import Tensor

from . import _native as N
from ._native import NativeError, call, ptr, stream
from .model import _error_word, attention, linear_ex


def _f32(t: Tensor) -> Tensor:
    return t if t.dtype == torch.float32 else t.float()


class _LinearFn(torch.autograd.Function):
    """``act(x @ W_pad^T * row_scale + b + residual)`` on the bound map ``m`` (a ``_Map``)."""

    @staticmethod
    def forward(ctx, x, w, b, residual, m, activation, row_scale, group, out_dtype):
        m.refresh(w, b)
        y = linear_ex(x, m.weight, m.bias, activation, row_scale=row_scale, residual=residual, residual_group=group,
                      out_dtype=out_dtype)
        if m.np_ != m.n:
            y = y[:, : m.n]
        ctx.save_for_backward(x, row_scale, residual)
        ctx.m, ctx.activation, ctx.group = m, activation, group
        ctx.has_b, ctx.w_dtype = b is not None, w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, row_scale, residual = ctx.saved_tensors
        m = ctx.m
        M, n = x.shape[0], m.n
        dev = x.device
        if ctx.activation == "gelu" and m.np_ == n and dy.dtype == torch.bfloat16:
            # the map recomputed with dy * GELU'(pre-activation) in its epilogue: bf16 out, no fp32 round trip
            dy = dy.contiguous()
            dpre = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
            call("pbg_linear_gelu_backward", M, n, x.shape[1], ptr(x), x.stride(0), ptr(m.weight), ptr(m.bias),
                 ptr(row_scale), ptr(residual), 0 if residual is None else residual.stride(0), ctx.group, ptr(dy), n,
                 ptr(dpre), n, ptr(_error_word(dev)), stream(dev))
        elif ctx.activation == "gelu":
            pre = linear_ex(x, m.weight, m.bias, None, row_scale=row_scale, residual=residual,
                            residual_group=ctx.group, out_dtype=torch.float32)
            dy = dy.contiguous()
            dpre = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
            call("pbg_gelu_backward", M, n, ptr(pre), pre.stride(0), ptr(dy), int(dy.dtype == torch.bfloat16),
                 dy.stride(0), ptr(dpre), n, stream(dev))
        else:
            dpre = dy
        operand = dpre if row_scale is None else dpre.float() * row_scale[:, None]
        operand = operand.to(torch.bfloat16).contiguous()
        w_rows = m.weight[:n]
        dx = torch.mm(operand, w_rows) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = torch.mm(operand.t(), x, out_dtype=torch.float32)[:, : m.k]
        db = dpre.sum(0, dtype=torch.float32) if ctx.has_b and ctx.needs_input_grad[2] else None
        dres = None
        if residual is not None and ctx.needs_input_grad[3]:
            dres = _f32(dpre)
            if ctx.group > 1:
                dres = dres.view(M // ctx.group, ctx.group, n).sum(1)
        return dx, dw, db, dres, None, None, None, None, None


def linear_train(m, rows: Tensor, activation: str | None = None, *, row_scale: Tensor | None = None,
                 residual: Tensor | None = None, residual_group: int = 1, out_dtype=torch.bfloat16) -> Tensor:
    """The map ``m`` over bf16 rows [M, kp] with its fp32 master weight and bias as autograd inputs."""

    w, b = m.source()
    if row_scale is not None:
        row_scale = row_scale.detach().float().contiguous()
    if residual is not None and residual.dtype != torch.float32:
        residual = residual.float()
    return _LinearFn.apply(rows.contiguous(), w, b, None if residual is None else residual.contiguous(), m, activation,
                           row_scale, residual_group, out_dtype)


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gain, bias, eps):
        rows, d = x.shape
        out = torch.empty((rows, d), dtype=torch.bfloat16, device=x.device)
        call("pbg_layernorm", rows, d, ptr(x), int(x.dtype == torch.bfloat16), ptr(gain), ptr(bias), eps,
             ctypes.c_void_p(out.data_ptr()), 1, d, stream(x.device))
        ctx.save_for_backward(x, gain)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, dy):
        x, gain = ctx.saved_tensors
        rows, d = x.shape
        dev = x.device
        dy = dy.contiguous()
        dx = torch.empty_like(x)
        blocks = int(N.lib().pbg_layernorm_backward_partials(rows, d))
        if blocks < 0:
            raise NativeError(f"layernorm backward does not take width {d}")
        partial = torch.empty(blocks, dtype=torch.float32, device=dev)
        call("pbg_layernorm_backward", rows, d, ptr(x), int(x.dtype == torch.bfloat16), d, ptr(gain), ctx.eps,
             ptr(dy), int(dy.dtype == torch.bfloat16), d, ptr(dx), int(dx.dtype == torch.bfloat16), d, ptr(partial),
             blocks, stream(dev))
        sums = partial.view(-1, 2, d).sum(0)
        return dx, sums[0], sums[1], None


def layernorm_train(x: Tensor, gain: Tensor, bias: Tensor, eps: float = 1e-5) -> Tensor:
    """LayerNorm over the last dimension, bf16 out, differentiable in x, gain and bias."""

    d = x.shape[-1]
    y = _LayerNormFn.apply(x.reshape(-1, d).contiguous(), gain, bias, eps)
    return y.view(*x.shape[:-1], d)


class _AttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, q_scale, key_bias, key_mask, heads):
        B, L, _ = qkv.shape
        lse = torch.empty((B, heads, L), dtype=torch.float32, device=qkv.device)
        out = attention(qkv, heads, q_scale, key_bias, key_mask, lse=lse)
        ctx.save_for_backward(qkv, q_scale, key_bias, key_mask, out, lse)
        ctx.heads = heads
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, q_scale, key_bias, key_mask, out, lse = ctx.saved_tensors
        H = ctx.heads
        B, L, _ = qkv.shape
        dev = qkv.device
        dout = dout.to(torch.bfloat16).contiguous()
        dqkv = torch.empty_like(qkv)
        delta = torch.empty((B, H, L), dtype=torch.float32, device=dev)
        partial = torch.empty((B, H, L), dtype=torch.float32, device=dev)
        bias = None if key_bias is None else key_bias.float().contiguous()
        mask = None if key_mask is None else key_mask.contiguous().view(torch.uint8)
        call("pbg_attention_backward", B, L, H, ptr(qkv), ptr(out), ptr(dout), ptr(lse), ptr(bias), ptr(mask),
             ptr(q_scale.detach().float().contiguous()), ptr(dqkv), ptr(delta), ptr(partial), stream(dev))
        return dqkv, partial.sum((0, 2)).to(q_scale.dtype), None, None, None


def attention_train(qkv: Tensor, heads: int, q_scale: Tensor, key_bias: Tensor | None,
                    key_mask: Tensor | None) -> Tensor:
    """The reach-biased attention core, differentiable in qkv and the per-head score scale."""

    kb = None if key_bias is None else key_bias.detach()
    km = None if key_mask is None else key_mask.detach()
    return _AttentionFn.apply(qkv.contiguous(), q_scale, kb, km, heads)


class _IncidenceCombineFn(torch.autograd.Function):
    """incidence.py:57-70 after the card contractions (``pbg_incidence_combine``): from source and
    overlap [B, P, R, d] (fp32) and the identical-row scale [B, R], the rows [oe | own] (bf16), oc
    (fp32) and the FamilyFFN features [oc^2 | oc * oe] (bf16), rows (b * P + p) * R + r; the backward
    is ``pbg_incidence_combine_backward``."""

    @staticmethod
    def forward(ctx, source, overlap, identical_scale):
        B, P, R, d = source.shape
        count, dev = B * P * R, source.device
        pair = torch.empty((count, 2 * d), dtype=torch.bfloat16, device=dev)
        other_card = torch.empty((count, d), dtype=torch.float32, device=dev)
        ffn = torch.empty((count, 2 * d), dtype=torch.bfloat16, device=dev)
        call("pbg_incidence_combine", B, P, R, d, ptr(source), ptr(overlap), ptr(identical_scale), ptr(pair), 2 * d, 0,
             d, ptr(other_card), ptr(ffn), P * R * 2 * d, 2 * d, 0, d, stream(dev))
        ctx.save_for_backward(source, overlap, identical_scale)
        return pair, other_card, ffn

    @staticmethod
    def backward(ctx, g_pair, g_other_card, g_ffn):
        source, overlap, identical_scale = ctx.saved_tensors
        B, P, R, d = source.shape
        d_source, d_overlap = torch.empty_like(source), torch.empty_like(source)
        flat = lambda g, dtype: None if g is None else g.to(dtype).contiguous()  # noqa: E731
        g_pair, g_other_card, g_ffn = flat(g_pair, torch.bfloat16), flat(g_other_card, torch.float32), flat(
            g_ffn, torch.bfloat16)
        call("pbg_incidence_combine_backward", B, P, R, d, ptr(source), ptr(overlap), ptr(identical_scale), ptr(g_pair),
             ptr(g_other_card), ptr(g_ffn), ptr(d_source), ptr(d_overlap), stream(source.device))
        return d_source, d_overlap, None


def incidence_combine_train(source: Tensor, overlap: Tensor, identical_scale: Tensor):
    """Differentiable ``pbg_incidence_combine``: ([oe | own] bf16, oc fp32, [oc^2 | oc oe] bf16) rows."""

    return _IncidenceCombineFn.apply(source.contiguous(), overlap.contiguous(),
                                     identical_scale.detach().float().contiguous())


def q_scale_of(theta: Tensor) -> Tensor:
    """primitives.py MHA: the score scale 1 / ((softplus(theta) + 0.5) sqrt(32)) of each head."""

    return 1.0 / ((torch.nn.functional.softplus(theta) + 0.5) * math.sqrt(32))


class FlatParameters:
    """Named parameters as leaf views of one flat fp32 master (in the given order); ``attach`` makes each
    leaf's ``.grad`` a view of one flat gradient buffer, so autograd accumulates the gradient in place
    there (shared parameters used by several forwards add up) and the optimizer and the gradient SUM
    see one flat vector."""

    def __init__(self, params: dict, device) -> None:
        dev = torch.device(device)
        self.names = list(params)
        self.shapes = {n: tuple(params[n].shape) for n in self.names}
        self.offsets: dict[str, int] = {}
        total = 0
        for n in self.names:
            self.offsets[n] = total
            total += math.prod(self.shapes[n])
        self.numel = total
        self.master = torch.empty(total, dtype=torch.float32, device=dev)
        self.leaves: dict[str, Tensor] = {}
        for n in self.names:
            view = self.view(self.master, n)
            view.copy_(params[n].detach().to(device=dev, dtype=torch.float32).reshape(view.shape))
            self.leaves[n] = view.requires_grad_(True)
        self.grad: Tensor | None = None

    def view(self, flat: Tensor, name: str) -> Tensor:
        a = self.offsets[name]
        shape = self.shapes[name]
        return flat[a: a + math.prod(shape)].view(shape)

    def attach(self, grad: Tensor) -> None:
        if grad.shape != (self.numel,) or grad.dtype != torch.float32:
            raise NativeError("the flat gradient must be fp32 [numel]")
        self.grad = grad
        for n, leaf in self.leaves.items():
            leaf.grad = self.view(grad, n)


_FIELDS = ("type_logits", "omega", "mu", "s", "iota")


class ModelLearnerStep:
    """The learner step over one batch per input family (pbg/core/training.py:336-424 with the queued
    model operation, pbg/games/poker/queued/model.py:403-415): for each batch the model's learner rows
    (the owner's sampled private row), the fused poker objective, and the backward of the objective's
    gradient through the network into the flat gradient; then one AdamW transition of the flat master.

    A batch is a dict with ``input_type``, ``model_input`` [S, F], ``sampled_private_state`` [S, P],
    ``owner`` [S], and the objective's ``mask``, ``action``, ``old_log_policy``, ``advantage_target``,
    ``old_value``, ``value_target``, ``controls`` and ``lane_weight``."""

    def __init__(self, model, *, lr: float = 3e-4, beta1: float = 0.9, beta2: float = 0.999, epsilon: float = 1e-8,
                 weight_decay: float = 0.0, grad_clip: float = 1.0) -> None:
        from .learner import PokerLearnerObjective
        from .optim import FlatAdam

        self.model = model
        self.flat = model.enable_training()
        self.adam = FlatAdam(self.flat.master, lr=lr, beta1=beta1, beta2=beta2, epsilon=epsilon, decay=weight_decay,
                             clip=grad_clip)
        self.flat.attach(self.adam.grad)
        self.objective = PokerLearnerObjective(self.flat.master.device)

    def gradient(self, batches: list) -> list:
        """Forward, objective and backward of every batch; the flat gradient lands in ``self.adam.grad``,
        cleared first (the AdamW transition leaves the clipped gradient there, and autograd adds into it)."""

        self.adam.grad.zero_()
        results = []
        for b in batches:
            evaluation = self.model.learner_operation(b["input_type"], b["model_input"], b["sampled_private_state"],
                                                      b["owner"])
            raw, value = evaluation.policy_raw, evaluation.value
            result, grads = self.objective(raw, b["mask"], b["action"], b["old_log_policy"], b["advantage_target"],
                                           value, b["old_value"], b["value_target"], b["controls"], b["lane_weight"])
            outputs = [raw[n] for n in _FIELDS] + [value]
            torch.autograd.backward(outputs, [grads[n].view_as(raw[n]) for n in _FIELDS] + [grads["value"].view_as(value)])
            results.append(result)
        return results

    def __call__(self, batches: list) -> list:
        results = self.gradient(batches)
        self.adam.step()
        return results
