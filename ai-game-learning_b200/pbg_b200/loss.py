"""Fused PPO loss backward for categorical decision rows.

``fused_ppo_backward`` is one HBM pass computing the learner objective of
pbg/core/learner.py:2021-2077 (clipped ratio, negative-advantage log cap,
entropy bonus) for the game-neutral categorical policy
(tests/categorical_policy_fixture.py:33-57), scaled per row by its
decision-mass weight, and writing d total / d logits.  The total is

    total = scale * sum_r w_r * (policy_row_r - c_ent * entropy_r) * inv_count

with ``inv_count = 1/N`` (the reference's lane mean, its local decision-mass
normalisation) or ``1/sum_global(w)`` when ``global_mass=True`` (the global
Z_{g,m}/Z scaling of the theory; the all-reduce of sum(w) happens before the
kernel on the caller's process group).
"""

from __future__ import annotations

from dataclasses import dataclass

import math

import torch
from torch import Tensor

import ctypes

from ._native import call, check, lib, ptr, stream

STATS = ("total", "policy", "entropy", "approximate_kl", "clip_count", "negative_cap_count", "weight_sum", "rows")


@dataclass(frozen=True)
class LossConfig:
    policy_clip: float = 0.2
    negative_advantage_ratio_cap: float | None = None
    entropy_coefficient: float = 0.01


class FusedPPOBackward:
    """Owns the small device buffers a call needs (controls, partials, stats)."""

    def __init__(self, rows: int, actions: int, device, config: LossConfig = LossConfig()) -> None:
        self.rows, self.actions = int(rows), int(actions)
        self.device = torch.device(device)
        self.config = config
        n = int(lib().pbg_ppo_partials_size(self.rows, self.actions))
        self.partials = torch.zeros(n, dtype=torch.float64, device=self.device)
        self.stats = torch.zeros(8, dtype=torch.float64, device=self.device)
        self.controls = torch.zeros(5, dtype=torch.float32, device=self.device)
        self.set_controls()

    def set_controls(self, *, scale: float = 1.0, inv_count: float | None = None) -> None:
        cap = self.config.negative_advantage_ratio_cap
        log_cap = math.inf if cap is None else math.log(cap)
        inv = (1.0 / self.rows if self.rows else 0.0) if inv_count is None else inv_count
        self.controls.copy_(torch.tensor([self.config.policy_clip, log_cap, self.config.entropy_coefficient,
                                          scale, inv], dtype=torch.float32))

    def __call__(self, logits: Tensor, mask: Tensor, action: Tensor, old_logp: Tensor, advantage: Tensor,
                 weight: Tensor, dlogits: Tensor | None = None) -> tuple[Tensor, Tensor]:
        N, A = logits.shape
        if (N, A) != (self.rows, self.actions):
            raise ValueError("loss rows/actions differ from the admitted shape")
        if logits.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("logits must be fp32 or bf16")
        if dlogits is None:
            dlogits = torch.empty_like(logits)
        call("pbg_ppo_categorical_backward", N, A, 1 if logits.dtype == torch.bfloat16 else 0, ptr(logits),
             ptr(mask.view(torch.uint8) if mask.dtype == torch.bool else mask), ptr(action), ptr(old_logp),
             ptr(advantage), ptr(weight), ptr(self.controls), ptr(dlogits), ptr(self.partials), ptr(self.stats),
             stream(logits.device))
        return dlogits, self.stats

    def bind(self, logits, mask, action, old_logp, advantage, weight, dlogits, *, max_ctas: int = 0
             ) -> BoundPPOBackward:
        """``max_ctas`` > 0 caps the persistent kernel's grid (SMs left to a collective on another stream)."""

        if tuple(logits.shape) != (self.rows, self.actions) or dlogits.shape != logits.shape:
            raise ValueError("loss rows/actions differ from the admitted shape")
        return BoundPPOBackward(self, logits, mask, action, old_logp, advantage, weight, dlogits, max_ctas)


class BoundPPOBackward:
    """A loss launch with its device pointers resolved once.

    Repeated steps over the same buffers (a learner's admitted batch slots)
    re-launch from cached arguments, so the host adds only the ctypes call;
    the launch also records cleanly into a CUDA graph (warm it up once first
    so one-time device set-up happens outside the capture).
    """

    def __init__(self, op: "FusedPPOBackward", logits, mask, action, old_logp, advantage, weight, dlogits,
                 max_ctas: int = 0):
        N, A = logits.shape
        tensors = (logits, mask.view(torch.uint8) if mask.dtype == torch.bool else mask, action, old_logp,
                   advantage, weight, op.controls, dlogits, op.partials, op.stats)
        for t in tensors:
            if not (t.is_cuda and t.is_contiguous()):
                raise ValueError("bound loss buffers must be contiguous CUDA tensors")
        self._keep = tensors
        self._fn = lib().pbg_ppo_categorical_backward_grid
        self._args = (N, A, 1 if logits.dtype == torch.bfloat16 else 0, *(ctypes.c_void_p(t.data_ptr()) for t in tensors),
                      int(max_ctas))
        self.stats = op.stats
        self.dlogits = dlogits

    def launch(self, stream=None) -> None:
        s = torch.cuda.current_stream() if stream is None else stream
        rc = self._fn(*self._args, ctypes.c_void_p(s.cuda_stream))
        if rc != 0:
            check(rc, "pbg_ppo_categorical_backward_grid")


class FusedPPOReadoutBackward:
    """The loss backward fused with the readout's weight gradient.

    The logits come from a readout ``x = h W^T + b`` (pbg/core/tensor_ops.py:25-38) over hidden rows
    ``h`` [N, d] (bf16, d = 64, 128 or 256) with A = 8 outputs.  One pass writes the bf16 dlogits
    (the values ``FusedPPOBackward`` writes) and the readout's ``dweight`` [8, d] and ``dbias`` [8]
    (fp32 sums of the bf16 dlogits against the hidden rows): the gradients autograd would form next
    with a separate weight-gradient GEMM that re-reads dlogits.
    """

    def __init__(self, rows: int, hidden: int, device, config: LossConfig = LossConfig()) -> None:
        self.rows, self.hidden = int(rows), int(hidden)
        self.device = torch.device(device)
        n = int(lib().pbg_ppo_readout_partials_size(self.rows, 8, self.hidden))
        if n < 0:
            raise ValueError("readout width must be 64, 128 or 256")
        self.loss = FusedPPOBackward(rows, 8, device, config)
        self.partials = torch.zeros(n, dtype=torch.float64, device=self.device)
        self.dweight = torch.zeros((8, self.hidden), dtype=torch.float32, device=self.device)
        self.dbias = torch.zeros(8, dtype=torch.float32, device=self.device)

    def set_controls(self, *, scale: float = 1.0, inv_count: float | None = None) -> None:
        self.loss.set_controls(scale=scale, inv_count=inv_count)

    def __call__(self, logits: Tensor, mask: Tensor, action: Tensor, old_logp: Tensor, advantage: Tensor,
                 weight: Tensor, hidden: Tensor, dlogits: Tensor | None = None):
        """Returns (dlogits, dweight, dbias, stats); the last three are this object's buffers."""

        if tuple(logits.shape) != (self.rows, 8) or logits.dtype != torch.bfloat16:
            raise ValueError("readout loss needs bf16 logits of the admitted [rows, 8] shape")
        if tuple(hidden.shape) != (self.rows, self.hidden) or hidden.dtype != torch.bfloat16:
            raise ValueError("hidden rows must be bf16 [rows, hidden]")
        if dlogits is None:
            dlogits = torch.empty_like(logits)
        call("pbg_ppo_readout_backward", self.rows, 8, ptr(logits),
             ptr(mask.view(torch.uint8) if mask.dtype == torch.bool else mask), ptr(action), ptr(old_logp),
             ptr(advantage), ptr(weight), ptr(self.loss.controls), ptr(hidden), self.hidden, ptr(dlogits),
             ptr(self.dweight), ptr(self.dbias), ptr(self.partials), ptr(self.loss.stats), stream(logits.device))
        return dlogits, self.dweight, self.dbias, self.loss.stats


def fused_ppo_backward(logits, mask, action, old_logp, advantage, weight, config: LossConfig = LossConfig(), *,
                       scale: float = 1.0, inv_count: float | None = None):
    op = FusedPPOBackward(logits.shape[0], logits.shape[1], logits.device, config)
    op.set_controls(scale=scale, inv_count=inv_count)
    d, stats = op(logits, mask, action, old_logp, advantage, weight)
    return d, stats.clone()
