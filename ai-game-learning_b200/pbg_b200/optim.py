"""Device-only flat Adam/AdamW transition (pbg/core/optimization.py:182-233).

The master parameters, gradients and both moments are single flat fp32
buffers (the reference's DenseGradientOwner layout, optimization.py:106-169)
so one fused kernel sequence updates the whole model.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ._native import call, lib, ptr, stream

CONTROL_NAMES = ("lr", "beta1", "beta2", "epsilon", "decay", "clip", "scale", "growth", "backoff", "interval")


class FlatAdam:
    def __init__(self, master: Tensor, *, lr=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, decay=0.0, clip=1.0,
                 scale=1.0, decoupled=True) -> None:
        if master.dtype != torch.float32 or master.ndim != 1 or not master.is_cuda:
            raise ValueError("flat masters must be CUDA fp32 [N]")
        self.master = master
        n = master.numel()
        dev = master.device
        self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        self.first = torch.zeros(n, dtype=torch.float32, device=dev)
        self.second = torch.zeros(n, dtype=torch.float32, device=dev)
        self.controls = torch.tensor([lr, beta1, beta2, epsilon, decay, clip, scale, 2.0, 0.5, 2000.0],
                                     dtype=torch.float32, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.int64, device=dev)
        self.partials = torch.zeros(int(lib().pbg_adam_partials_size(n)), dtype=torch.float64, device=dev)
        self.report = torch.zeros(8, dtype=torch.float64, device=dev)
        self.decoupled = bool(decoupled)

    def step(self) -> Tensor:
        """Apply one transition from ``self.grad``; returns the device report."""

        call("pbg_adam_step", self.master.numel(), ptr(self.master), ptr(self.grad), ptr(self.first),
             ptr(self.second), ptr(self.controls), ptr(self.step_count), int(self.decoupled), ptr(self.partials),
             ptr(self.report), stream(self.master.device))
        return self.report
