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
    def __init__(self, group=None, nvls: "NVLSFlatSum | None" = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("DistributedSUM requires an initialised process group")
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.nvls = nvls  # gradients living in this buffer are summed by the NVLS kernel

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
        if self.nvls is not None and gradients.data_ptr() == self.nvls.buffer.data_ptr() \
                and gradients.numel() == self.nvls.numel:
            self.nvls.sum_()
        else:
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


class NVLSFlatSum:
    """A flat fp32 gradient buffer summed across ranks through NVLink SHARP.

    The buffer lives in torch symmetric memory bound to a multicast object;
    ``sum_()`` launches libpbgb200's multimem all-reduce (each rank reduces
    its 1/world slice in the switch and multicasts the result), replacing the
    NCCL SUM of replica.py:352-362 for this buffer.  Raises if the fabric has
    no multicast support; every rank must call ``sum_()`` in the same order.
    """

    def __init__(self, numel: int, device, group=None) -> None:
        import ctypes

        import torch.distributed._symmetric_memory as symm

        from ._native import lib

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if numel % (4 * self.world):
            raise ValueError("NVLS SUM needs numel to be a multiple of 4 * world_size")
        self.buffer = symm.empty(numel, dtype=torch.float32, device=device)
        self.buffer.zero_()
        self.handle = symm.rendezvous(self.buffer, self.group)
        if int(self.handle.multicast_ptr) == 0:
            raise RuntimeError("this fabric exposes no NVLS multicast object")
        self.pad_bytes = int(self.handle.signal_pad_size)
        if self.pad_bytes < int(lib().pbg_nvls_signal_bytes()):
            raise RuntimeError("symmetric-memory signal pad is smaller than the NVLS barrier needs")
        base = int(self.handle.buffer_ptrs[self.rank])
        self.multicast = ctypes.c_void_p(int(self.handle.multicast_ptr) + (self.buffer.data_ptr() - base))
        self.pads = ctypes.c_void_p(int(self.handle.signal_pad_ptrs_dev))
        self.error = torch.zeros(1, dtype=torch.int32, device=device)
        self.numel = numel
        # the barrier slots must start at zero on every rank before the first call
        pad = self.handle.get_signal_pad(self.rank, (self.pad_bytes // 4,), dtype=torch.int32)
        pad.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def sum_(self, stream=None) -> torch.Tensor:
        """In-place SUM of ``buffer`` over all ranks (stream-ordered, no host sync)."""

        from ._native import call, ptr

        s = torch.cuda.current_stream() if stream is None else stream
        call("pbg_nvls_allreduce_sum_f32", self.numel, self.multicast, self.pads, self.pad_bytes, self.rank,
             self.world, ptr(self.error), ctypes_stream(s))
        return self.buffer

    def check(self) -> None:
        """Raise if any barrier wait of an earlier sum_() ran out (synchronises)."""

        if int(self.error.item()) != 0:
            raise RuntimeError("an NVLS all-reduce barrier timed out on this rank")


def ctypes_stream(s):
    import ctypes

    return ctypes.c_void_p(s.cuda_stream)
