"""Dense layers of the poker policy/value model on the tensor cores.

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

from ._native import NativeError, call, ptr, stream

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


__all__ = ["FFN", "Linear", "linear", "pipeline_error"]
