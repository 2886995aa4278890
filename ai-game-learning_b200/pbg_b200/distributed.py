"""Rank-common gradient SUM and agreement (pbg/core/replica.py:321-379).

``DistributedSUM`` keeps the reference's duck type (agree_active,
agree_failures, sum_gradients, barrier, maximum_steps) over a
torch.distributed process group: NCCL on GPUs, gloo in the CPU tests.  The
gradient SUM is one all-reduce of the flat fp32 buffer [K, N].  The agreement
scalars of one optimizer step (active lanes, failed lanes, the step budget)
travel together in ONE int32 MAX all-reduce (``agree``): a lane's MIN over
ranks is recovered as 1 - MAX(1 - active).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import Tensor


class ReplicaError(RuntimeError):
    """Ranks disagree on replica state (replica.py: ReplicaError)."""


class DistributedSUM:
    def __init__(self, group=None, nvls: "NVLSFlatSum | None" = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("DistributedSUM requires an initialised process group")
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.nvls = nvls  # gradients living in this buffer are summed by the NVLS kernel

    def _max(self, packed: Tensor) -> Tensor:
        dist.all_reduce(packed, op=dist.ReduceOp.MAX, group=self.group)
        return packed

    def agree(self, active: Tensor, failed: Tensor | None = None, local_steps: int = 0) -> tuple[Tensor, int]:
        """One step's agreement in one MAX all-reduce.

        Packs ``[active, 1 - active, failed, steps]`` as int32; raises
        ``ReplicaError`` when the ranks selected different active lanes
        (replica.py:332-345), and returns the lanes failed on any rank
        (:347-350) and the rank-common step budget (:369-379).  One host read.
        """

        if isinstance(local_steps, bool) or local_steps < 0:
            raise ValueError("local optimizer step count must be nonnegative")
        k = active.numel()
        if failed is None:
            failed = torch.zeros_like(active)
        if failed.shape != active.shape:
            raise ValueError("failure and active masks must have one entry per lane")
        a = active.reshape(-1).to(torch.int32)
        packed = torch.cat((a, 1 - a, failed.reshape(-1).to(torch.int32),
                            torch.tensor([int(local_steps)], dtype=torch.int32, device=active.device)))
        out = self._max(packed).cpu()
        any_active, not_all = out[:k], out[k:2 * k]
        if not torch.equal(any_active, 1 - not_all):
            raise ReplicaError("distributed ranks selected asymmetric active lanes")
        failures = out[2 * k:3 * k].bool().reshape(active.shape).to(active.device)
        return failures, int(out[3 * k])

    def agree_active(self, active: Tensor) -> Tensor:
        """replica.py:332-345: raise unless every rank selected the same active lanes."""

        self.agree(active)
        return active.bool()

    def agree_failures(self, failed: Tensor) -> Tensor:
        """replica.py:347-350: a lane failed if it failed on any rank."""

        flags = failed.to(torch.uint8).clone()
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.group)
        return flags.bool()

    def sum_gradients(self, gradients: Tensor, active: Tensor, *, agreed: bool = False) -> Tensor:
        """replica.py:352-362: zero inactive lanes, then one SUM all-reduce.

        ``agreed=True`` skips the active-lane agreement when the caller has
        already run ``agree`` for this step (no host read then).
        """

        if gradients.dtype != torch.float32 or gradients.ndim != 2 or active.shape != gradients.shape[:1]:
            raise ValueError("gradient SUM requires fp32 [K,N] and one active flag per lane")
        if not agreed:
            self.agree(active)
        gradients.masked_fill_(~active.bool()[:, None], 0.0)
        if self.nvls is not None and gradients.data_ptr() == self.nvls.buffer.data_ptr() \
                and gradients.numel() == self.nvls.numel:
            self.nvls.raise_if_failed()
            self.nvls.sum_()
        else:
            dist.all_reduce(gradients, op=dist.ReduceOp.SUM, group=self.group)
        return gradients

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    def maximum_steps(self, steps: int, device) -> int:
        """replica.py:369-379: rank-common optimizer budget."""

        if isinstance(steps, bool) or steps < 0:
            raise ValueError("local optimizer step count must be nonnegative")
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
        self._host_error = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._copied = torch.cuda.Event()
        self._copied.record()
        self.numel = numel
        # the barrier slots must start at zero on every rank before the first call
        pad = self.handle.get_signal_pad(self.rank, (self.pad_bytes // 4,), dtype=torch.int32)
        pad.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def sum_(self, stream=None) -> torch.Tensor:
        """In-place SUM of ``buffer`` over all ranks (stream-ordered, no host sync).

        The error word is sticky: once a barrier wait of some call ran out,
        every later launch returns at entry without touching the buffer or
        the signal pads, so a late peer signal can never release a later
        barrier early.  After each launch the word is copied (asynchronously)
        to pinned host memory; ``raise_if_failed`` reads the newest copy that
        has landed without waiting for the GPU.
        """

        from ._native import call, ptr

        s = torch.cuda.current_stream() if stream is None else stream
        call("pbg_nvls_allreduce_sum_f32", self.numel, self.multicast, self.pads, self.pad_bytes, self.rank,
             self.world, ptr(self.error), ctypes_stream(s))
        if not torch.cuda.is_current_stream_capturing():
            with torch.cuda.stream(s):
                self._host_error.copy_(self.error, non_blocking=True)
                self._copied.record(s)
        return self.buffer

    def sum_range_(self, start: int, count: int, stream=None, max_ctas: int = 0) -> torch.Tensor:
        """In-place SUM of ``buffer[start:start + count]`` (a bucket; both multiples of 4 * world).

        Buckets go through the same signal pads, so launch them on ONE stream (in the same order on
        every rank); a bucket may start while other work on this GPU is still running.  ``max_ctas``
        > 0 caps the kernel's grid, so it runs beside compute that holds the other SMs.
        """

        from ._native import call, ptr

        if start % (4 * self.world) or count % (4 * self.world) or count <= 0 or start + count > self.numel:
            raise ValueError("NVLS bucket bounds must be positive multiples of 4 * world_size inside the buffer")
        s = torch.cuda.current_stream() if stream is None else stream
        mc = ctypes.c_void_p(self.multicast.value + 4 * start)
        call("pbg_nvls_allreduce_sum_f32_grid", count, mc, self.pads, self.pad_bytes, self.rank, self.world,
             ptr(self.error), int(max_ctas), ctypes_stream(s))
        if not torch.cuda.is_current_stream_capturing():
            with torch.cuda.stream(s):
                self._host_error.copy_(self.error, non_blocking=True)
                self._copied.record(s)
        return self.buffer[start:start + count]

    def raise_if_failed(self) -> None:
        """Raise if an earlier sum_() reported a barrier timeout (no host sync).

        Reads the pinned copy of the error word made after the newest
        sum_() whose copy has completed; a call still in flight is seen by a
        later check.
        """

        if self._copied.query() and int(self._host_error[0]) != 0:
            raise RuntimeError("an NVLS all-reduce barrier timed out on this rank; the SUM is disabled "
                               "until reset()")

    def check(self) -> None:
        """Raise if any barrier wait of an earlier sum_() ran out (synchronises)."""

        if int(self.error.item()) != 0:
            raise RuntimeError("an NVLS all-reduce barrier timed out on this rank")

    def reset(self) -> None:
        """Clear the error word and this rank's signal pad (collective: every rank calls it).

        Synchronises the device and the group first, so no launch is in
        flight on any rank while the slots are cleared.
        """

        torch.cuda.synchronize(self.buffer.device)
        dist.barrier(group=self.group)
        pad = self.handle.get_signal_pad(self.rank, (self.pad_bytes // 4,), dtype=torch.int32)
        pad.zero_()
        self.error.zero_()
        self._host_error.zero_()
        torch.cuda.synchronize(self.buffer.device)
        dist.barrier(group=self.group)


def ctypes_stream(s):
    import ctypes

    return ctypes.c_void_p(s.cuda_stream)
