"""Dense layers of the poker policy/value model on the tensor cores.

``attention`` is the reach-biased self-attention core of the model's MHA
(pbg/games/poker/model/primitives.py:63-283) on the tensor cores; ``MHA``
composes it with the two projections.

``linear`` is the affine map of pbg/core/tensor_ops.py ``Linear`` (weight
``[out, in]``, bias ``[out]``) as used by the model's FFN
(pbg/games/poker/model/primitives.py:35-60: ``w2(gelu(w1(x)))``) and by the
attention projections (primitives.py:97-117: ``w_qkv``, ``w_o``), computed by
``pbg_linear_bf16``: bf16 operands, fp32 accumulation in tensor memory, bias
and GELU fused into the epilogue.  There is no fallback: shapes the kernel
does not take raise.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from ._native import NativeError, call, ptr, rows_ptr, stream

ACTIVATIONS = {None: 0, "none": 0, "gelu": 1}
_ERROR: dict[int, Tensor] = {}


def _error_word(device: torch.device) -> Tensor:
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _ERROR.get(index)
    if word is None:
        word = _ERROR[index] = torch.zeros(1, dtype=torch.int32, device=device)
    return word


def pipeline_error(device=None) -> int:
    """The sticky pipeline-timeout code of the device's linear launches (0 = none); synchronises."""

    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return int(_error_word(device).item())


def linear(x: Tensor, weight: Tensor, bias: Tensor | None = None, activation: str | None = None,
           out: Tensor | None = None) -> Tensor:
    """``act(x @ weight.T + bias)`` over the last dimension of ``x`` (bf16 in and out)."""

    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise NativeError("linear takes bf16 inputs and weights")
    if weight.ndim != 2 or x.shape[-1] != weight.shape[1]:
        raise NativeError("linear: x [..., in] and weight [out, in] do not match")
    if bias is not None and (bias.dtype != torch.float32 or bias.shape != (weight.shape[0],)):
        raise NativeError("linear: bias must be float32 [out]")
    n, k = weight.shape
    rows = x.reshape(-1, k)
    if not rows.is_contiguous():
        rows = rows.contiguous()
    w = weight.contiguous()
    if out is None:
        out = torch.empty((*x.shape[:-1], n), dtype=torch.bfloat16, device=x.device)
    call("pbg_linear_bf16", rows.shape[0], n, k, ptr(rows), ptr(w), ptr(bias), ptr(out),
         ACTIVATIONS[activation], ptr(_error_word(x.device)), stream(x.device))
    return out


def linear_ex(x: Tensor, weight: Tensor, bias: Tensor | None = None, activation: str | None = None, *,
              row_scale: Tensor | None = None, residual: Tensor | None = None, residual_group: int = 1,
              out: Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """``act(x @ weight.T * row_scale[:, None] + bias + residual)`` on ``pbg_linear_ex``.

    ``x`` bf16 ``[M, K]`` and ``out`` ``[M, N]`` may be column slices of wider buffers (rows
    contiguous, any row stride); ``residual`` fp32 ``[M / residual_group, N]`` likewise, row m of
    the output adding residual row ``m // residual_group``; ``row_scale`` fp32 ``[M]``.  The output
    is bf16 or fp32 (``out_dtype``, or ``out``'s dtype).
    """

    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or x.ndim != 2:
        raise NativeError("linear_ex takes a bf16 matrix x and bf16 weights")
    n, k = weight.shape
    m = x.shape[0]
    if x.shape[1] != k:
        raise NativeError("linear_ex: x [M, in] and weight [out, in] do not match")
    if bias is not None and (bias.dtype != torch.float32 or bias.shape != (n,)):
        raise NativeError("linear_ex: bias must be float32 [out]")
    if row_scale is not None and (row_scale.dtype != torch.float32 or row_scale.shape != (m,)):
        raise NativeError("linear_ex: row_scale must be float32 [M]")
    if residual is not None and (residual.dtype != torch.float32 or residual_group < 1 or m % residual_group
                                 or residual.shape != (m // residual_group, n)):
        raise NativeError("linear_ex: residual must be float32 [M / residual_group, out]")
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    if out.shape != (m, n) or out.dtype not in (torch.bfloat16, torch.float32):
        raise NativeError("linear_ex: out must be [M, out] bf16 or fp32")
    call("pbg_linear_ex", m, n, k, rows_ptr(x), x.stride(0), ptr(weight.contiguous()), ptr(bias), ptr(row_scale),
         rows_ptr(residual), 0 if residual is None else residual.stride(0), residual_group, rows_ptr(out), out.stride(0),
         int(out.dtype == torch.float32), ACTIVATIONS[activation], ptr(_error_word(x.device)), stream(x.device))
    return out


class Linear:
    """Affine map with the reference's parameter layout (weight ``[out, in]`` bf16, bias ``[out]`` fp32)."""

    def __init__(self, weight: Tensor, bias: Tensor | None = None) -> None:
        self.weight = weight.to(torch.bfloat16).contiguous()
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()

    def __call__(self, x: Tensor, activation: str | None = None) -> Tensor:
        return linear(x, self.weight, self.bias, activation)


class FFN:
    """primitives.py:35-60 ``FFN``: ``w2(gelu(w1(x)))``, GELU fused into the first map's epilogue."""

    def __init__(self, w1: Linear, w2: Linear) -> None:
        if w1.weight.shape[0] != w2.weight.shape[1]:
            raise NativeError("FFN: hidden widths do not match")
        self.w1, self.w2 = w1, w2

    def __call__(self, x: Tensor) -> Tensor:
        return self.w2(self.w1(x, "gelu"))


def attention(qkv: Tensor, heads: int, q_scale: Tensor, key_bias: Tensor | None = None,
              key_mask: Tensor | None = None, lse: Tensor | None = None) -> Tensor:
    """Self-attention core of primitives.py MHA for heads of width 32 (pbg_attention_bf16).

    ``qkv`` bf16 ``[B, L, 3 * heads * 32]`` (the fused in-projection's output),
    ``q_scale`` fp32 ``[heads]`` = 1 / (temperature * sqrt(32)), ``key_bias``
    fp32 ``[B, L]``, ``key_mask`` bool ``[B, L]``.  Returns merged heads, bf16
    ``[B, L, heads * 32]``; with ``lse`` (fp32 ``[B, heads, L]``) also each
    row's base-2 log-sum-exp of its logits (the backward's input).
    """

    if qkv.dtype != torch.bfloat16 or qkv.ndim != 3 or qkv.shape[2] != 3 * heads * 32:
        raise NativeError("attention takes bf16 qkv [B, L, 3 * heads * 32]")
    batch, length, _ = qkv.shape
    qkv = qkv.contiguous()
    if key_bias is not None and (key_bias.dtype != torch.float32 or key_bias.shape != (batch, length)):
        raise NativeError("key_bias must be float32 [B, L]")
    if key_mask is not None and (key_mask.dtype != torch.bool or key_mask.shape != (batch, length)):
        raise NativeError("key_mask must be bool [B, L]")
    scale = q_scale.to(device=qkv.device, dtype=torch.float32).contiguous()
    if scale.shape != (heads,):
        raise NativeError("q_scale must hold one value per head")
    out = torch.empty((batch, length, heads * 32), dtype=torch.bfloat16, device=qkv.device)
    mask = None if key_mask is None else key_mask.contiguous().view(torch.uint8)
    bias = None if key_bias is None else key_bias.contiguous()
    if lse is None:
        call("pbg_attention_bf16", batch, length, heads, ptr(qkv), ptr(bias), ptr(mask), ptr(scale), ptr(out),
             ptr(_error_word(qkv.device)), stream(qkv.device))
        return out
    if lse.dtype != torch.float32 or lse.shape != (batch, heads, length) or not lse.is_contiguous():
        raise NativeError("lse must be contiguous float32 [B, heads, L]")
    call("pbg_attention_bf16_lse", batch, length, heads, ptr(qkv), ptr(bias), ptr(mask), ptr(scale), ptr(out),
         ptr(lse), ptr(_error_word(qkv.device)), stream(qkv.device))
    return out


class MHA:
    """primitives.py:63-283 MHA (self-attention) with the reference's parameters.

    ``w_qkv`` / ``w_o`` are Linear maps (weight ``[3d, d]`` / ``[d, d]``),
    ``theta`` ``[heads]`` gives the learned temperature softplus(theta) + 0.5.
    """

    def __init__(self, w_qkv: Linear, w_o: Linear, theta: Tensor, heads: int) -> None:
        d = w_o.weight.shape[0]
        if d != heads * 32 or w_qkv.weight.shape != (3 * d, d):
            raise NativeError("MHA: this build's attention core takes heads of width 32")
        self.w_qkv, self.w_o, self.heads = w_qkv, w_o, heads
        temperature = torch.nn.functional.softplus(theta.float()) + 0.5
        self.q_scale = (1.0 / (temperature * 32 ** 0.5)).contiguous()

    def forward_biased(self, x: Tensor, key_bias: Tensor | None, key_mask: Tensor | None) -> Tensor:
        merged = attention(self.w_qkv(x), self.heads, self.q_scale.to(x.device), key_bias, key_mask)
        return self.w_o(merged)

    __call__ = forward_biased


__all__ = ["FFN", "Linear", "MHA", "attention", "linear", "pipeline_error"]
