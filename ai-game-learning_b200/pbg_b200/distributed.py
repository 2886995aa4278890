"""Rank-common gradient SUM and agreement (pbg/core/replica.py:321-379).

``DistributedSUM`` keeps the reference's duck type (agree_active,
agree_failures, sum_gradients, barrier, maximum_steps) over a
torch.distributed process group: NCCL on GPUs, gloo in the CPU tests.  The
gradient SUM is one all-reduce of the flat fp32 buffer [K, N]; the small
agreement flags are single MIN/MAX all-reduces, as in the reference.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


class DistributedSUM:
    def __init__(self, group=None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("DistributedSUM requires an initialised process group")
        self.group = group
        self.world_size = dist.get_world_size(group)

    def agree_active(self, active: Tensor) -> Tensor:
        """replica.py:332-345: lanes active on every rank; raise on disagreement."""

        low = active.to(torch.uint8).clone()
        high = low.clone()
        dist.all_reduce(low, op=dist.ReduceOp.MIN, group=self.group)
        dist.all_reduce(high, op=dist.ReduceOp.MAX, group=self.group)
        if not torch.equal(low, high):
            raise RuntimeError("ranks disagree on active replica lanes")
        return low.bool()

    def agree_failures(self, failed: Tensor) -> Tensor:
        """replica.py:347-350: a lane failed if it failed on any rank."""

        flags = failed.to(torch.uint8).clone()
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.group)
        return flags.bool()

    def sum_gradients(self, gradients: Tensor, active: Tensor) -> Tensor:
        """replica.py:352-362: zero inactive lanes, then one SUM all-reduce."""

        if gradients.dtype != torch.float32 or gradients.ndim != 2:
            raise ValueError("gradient SUM requires fp32 [K,N]")
        agreed = self.agree_active(active)
        gradients.mul_(agreed.to(gradients.dtype)[:, None])
        dist.all_reduce(gradients, op=dist.ReduceOp.SUM, group=self.group)
        return gradients

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    def maximum_steps(self, steps: int, device) -> int:
        """replica.py:369-379: rank-common optimizer budget."""

        value = torch.tensor([int(steps)], dtype=torch.int64, device=device)
        dist.all_reduce(value, op=dist.ReduceOp.MAX, group=self.group)
        return int(value.item())

    def global_sum(self, value: Tensor) -> Tensor:
        """All-reduced SUM of a small tensor (the global decision mass Z)."""

        out = value.clone()
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out
