"""Layered lambda-return targets over a topology forest.

``run_layers`` has the argument list and result of the reference's queued
layer operator (pbg/core/csrc/layered_targets.cu:311-411, loaded by
pbg/core/cuda_layer.py:13 and called from pbg/core/targets.py:640): node and
child column tensors, per-partition arena tensors, the conversion table and
the scalar shape arguments in, the per-lane ``failure_min`` (int32,
INT32_MAX = lane published) out.  The difference is the launch: every layer
runs inside ONE cooperative kernel with a grid barrier between layers,
instead of one kernel per layer queued from a host loop.

``LayeredTargets`` builds the device pointer tables once; ``launch`` then
enqueues the single kernel with no allocation or host copy, so a caller can
replay it per iteration.  ``run_layers`` keeps the last few bindings keyed by
the arguments' addresses, layer offsets and scalars, so repeated calls over
persistent arenas (the reference executor's pattern) skip the table upload.
"""

from __future__ import annotations

import ctypes
import math
from collections import OrderedDict
from typing import Sequence

import numpy as np
import torch
from torch import Tensor

from ._native import NativeError, TargetChildren, TargetNodes, TargetTables, call, lib, stream

INT32_MAX = 2**31 - 1
BARRIER_TIMEOUT = -2  # failure_min value of every lane when a grid barrier wait ran out

NODE_COLUMNS = ("replica", "child_begin", "child_count", "destination_row", "input_type", "output_type",
                "owner_slot", "nominal_degree", "target_degree", "sigma_head_row", "sigma_target_row",
                "action_begin")
CHILD_COLUMNS = ("source_row", "source_type", "path", "multiplier")


class TargetError(RuntimeError):
    """Invalid layered-target arguments (pbg/core/targets.py:40)."""


def _lambda(value: float) -> float:
    result = float(value)
    if not math.isfinite(result) or not 0.0 <= result <= 1.0:
        raise TargetError("lambda must be finite and lie in [0, 1]")
    return result


def conversion_table(widths: Sequence[int], maps: dict[tuple[int, int], Sequence[int]]) -> Tensor:
    """[outputs, outputs, max_width] int32 source component -> destination component (-1 none).

    ``maps[(source, destination)][h]`` names the destination class of source
    component h (pbg/core/targets.py:88-94 ConversionMap.destination_index);
    identity rows are filled for source == destination, as
    pbg/core/targets.py:609-626 does.
    """

    n = len(widths)
    width = max(widths)
    table = torch.full((n, n, width), -1, dtype=torch.int32)
    for s in range(n):
        table[s, s, : widths[s]] = torch.arange(widths[s], dtype=torch.int32)
    for (s, d), index in maps.items():
        if len(index) != widths[s]:
            raise TargetError("conversion map does not cover its source width")
        if any(i < 0 or i >= widths[d] for i in index):
            raise TargetError("conversion destination index is out of range")
        table[s, d, : widths[s]] = torch.tensor(list(index), dtype=torch.int32)
    return table


class LayeredTargets:
    """One bound forest: pointer tables and columns resident on the device."""

    def __init__(self, layer_ptr: Tensor, nodes: Sequence[Tensor], children: Sequence[Tensor],
                 work0, work1, trace, cost, delta, head_v, head_t, head_c, sigma_v, sigma_t, sigma_c,
                 action_p, action_a, conversion: Tensor, work_cap: Sequence[int], head_cap: Sequence[int],
                 width: Sequence[int], n_replica: int, input_count: int, output_count: int,
                 action_partition_count: int, p_train: int, max_width: int, lambda_: float, sampled: bool,
                 branched: bool) -> None:
        if len(nodes) != len(NODE_COLUMNS) or len(children) != len(CHILD_COLUMNS):
            raise TargetError("node/child column count differs from the layer-plan schema")
        device = nodes[0].device
        if device.type != "cuda":
            raise TargetError("queued targets require CUDA")
        self.device = device
        for t in list(nodes) + list(children[:3]):
            if t.device != device or t.dtype != torch.int32 or not t.is_contiguous():
                raise TargetError("layer-plan columns must be contiguous int32 on one CUDA device")
        if children[3].dtype != torch.float32 or children[3].device != device:
            raise TargetError("cost multipliers must be float32 on the plan's device")
        self.lambda_ = _lambda(lambda_)
        counts = dict(output_count=(work0, work1, trace, cost, delta), input_count=(head_v, head_t, head_c))
        for name, groups in counts.items():
            n = output_count if name == "output_count" else input_count
            for g in groups:
                if len(g) != n:
                    raise TargetError(f"arena table length differs from {name}")
        for g in (sigma_v, sigma_t, sigma_c):
            if len(g) != n_replica * input_count:
                raise TargetError("sigma tables must hold n_replica * input_count entries")
        for g in (action_p, action_a):
            if len(g) != n_replica * action_partition_count:
                raise TargetError("action tables must hold n_replica * action_partition_count entries")
        if not (len(work_cap) == len(width) == output_count and len(head_cap) == input_count):
            raise TargetError("capacity/width lists differ from the partition counts")
        if max_width != max(width) or conversion.numel() != output_count * output_count * max_width:
            raise TargetError("conversion table shape differs from [outputs, outputs, max_width]")

        # every pointer table, the integer tables and the layer offsets in one pinned host buffer, one
        # copy to the device; like the reference's pointer tables, entries are the tensors' addresses
        self._arenas = [list(g) for g in (work0, work1, trace, cost, delta, head_v, head_t, head_c, sigma_v,
                                          sigma_t, sigma_c, action_p, action_a)]  # keep the arenas alive
        for g in self._arenas:
            if g and (g[0].device != device or g[0].dtype != torch.float32):
                raise TargetError("arena tensors must be float32 on the plan's device")
        lengths = [len(g) for g in self._arenas]
        flat = [p for g in self._arenas for p in map(_DATA_PTR, g)]
        ints = [int(v) for v in work_cap] + [int(v) for v in head_cap] + [int(v) for v in width]
        lp = layer_ptr.to(dtype=torch.int32).flatten().tolist() if layer_ptr.device.type == "cpu" else None
        small = ints + (lp or [])
        host = torch.empty(len(flat) + (len(small) + 1) // 2, dtype=torch.int64, pin_memory=True)
        host.numpy()[: len(flat)] = flat
        host.numpy()[len(flat):].view(np.int32)[: len(small)] = small
        self._table_block = host.to(device, non_blocking=True)
        self._host_block = host  # pinned source of the asynchronous copy
        self._tables, offset = [], 0
        for n in lengths:
            self._tables.append(self._table_block[offset: offset + n])
            offset += n
        int_block = self._table_block[offset:].view(torch.int32)
        n_out, n_in = len(work_cap), len(head_cap)
        self._ints = [int_block[:n_out], int_block[n_out: n_out + n_in],
                      int_block[n_out + n_in: 2 * n_out + n_in],
                      conversion.to(device=device, dtype=torch.int32).contiguous().flatten()]
        if lp is not None:
            self.layer_ptr = int_block[len(ints): len(ints) + len(lp)]
        else:
            self.layer_ptr = layer_ptr.to(device=device, dtype=torch.int32).contiguous()
        self.layers = int(self.layer_ptr.numel()) - 1
        if self.layers < 0:
            raise TargetError("layer_ptr must hold layers + 1 offsets")
        self.nodes = [t.contiguous() for t in nodes]
        self.children = [t.contiguous() for t in children]
        # failure_min [n_replica] (written by the kernel), then the persistent workspace (zeroed once)
        words = int(lib().pbg_layered_targets_workspace_words(int(n_replica)))
        self._words = torch.zeros(n_replica + words, dtype=torch.int32, device=device)
        self.failure_min = self._words[:n_replica]
        self.workspace = self._words[n_replica:]
        self.shape = (int(n_replica), int(input_count), int(output_count), int(action_partition_count),
                      int(p_train), int(max_width))
        self.sampled, self.branched = bool(sampled), bool(branched)
        self._args = self._bind()

    def _bind(self) -> tuple:
        addr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        nd = TargetNodes(*[addr(t) for t in self.nodes])
        ch = TargetChildren(*[addr(t) for t in self.children])
        tb = TargetTables(*[addr(t) for t in self._tables], *[addr(t) for t in self._ints])
        n_replica, input_count, output_count, action_count, p_train, max_width = self.shape
        return (addr(self.layer_ptr), self.layers, nd, ch, tb, n_replica, input_count, output_count, action_count,
                p_train, max_width, ctypes.c_float(self.lambda_), int(self.sampled), int(self.branched))

    def launch(self, cuda_stream=None, failure_out: Tensor | None = None) -> Tensor:
        """Enqueue the single cooperative launch; returns ``failure_min`` (device int32 [n_replica]).

        ``failure_out`` receives the result instead of the binding's own
        buffer (the kernel initialises it, no clearing needed).  Launches of
        one binding must be ordered on one stream: they share the
        workspace (grid-barrier words and failure codes).
        """

        out = self.failure_min if failure_out is None else failure_out
        if out.device != self.device or out.dtype != torch.int32 or out.numel() != self.shape[0]:
            raise TargetError("failure_out must be int32 [n_replica] on the plan's device")
        s = stream(self.device) if cuda_stream is None else ctypes.c_void_p(cuda_stream)
        call("pbg_layered_targets", *self._args, ctypes.c_void_p(out.data_ptr()),
             ctypes.c_void_p(self.workspace.data_ptr()), s)
        return out

    def reset_barrier(self) -> None:
        """Clear the workspace after a launch that reported BARRIER_TIMEOUT."""

        self.workspace.zero_()


def run_layers(layer_ptr_cpu: Tensor, nodes: Sequence[Tensor], children: Sequence[Tensor], work0, work1, trace,
               cost, delta, head_v, head_t, head_c, sigma_v, sigma_t, sigma_c, action_p, action_a,
               conversion: Tensor, work_cap, head_cap, width, n_replica: int, input_count: int, output_count: int,
               action_partition_count: int, p_train: int, max_width: int, lambda_: float, sampled: bool,
               branched: bool) -> Tensor:
    """pbg/core/csrc/layered_targets.cu:311 run_layers: the same arguments, the same ``failure_min`` result."""

    if layer_ptr_cpu.device.type != "cpu":
        raise TargetError("layer_ptr must be CPU")
    groups = (work0, work1, trace, cost, delta, head_v, head_t, head_c, sigma_v, sigma_t, sigma_c, action_p, action_a)
    # a binding depends only on addresses, the layer offsets, the conversion table and the scalars
    conv_key = (conversion.data_ptr(),) if (conversion.is_cuda and conversion.dtype == torch.int32
                                             and conversion.is_contiguous()) else tuple(conversion.flatten().tolist())
    key = (nodes[0].device.index, tuple(layer_ptr_cpu.tolist()), tuple(map(_DATA_PTR, nodes)),
           tuple(map(_DATA_PTR, children)), tuple(tuple(map(_DATA_PTR, g)) for g in groups), conv_key,
           tuple(work_cap), tuple(head_cap), tuple(width), n_replica, input_count, output_count,
           action_partition_count, p_train, max_width, float(lambda_), bool(sampled), bool(branched))
    bound = _BINDINGS.get(key)
    if bound is None:
        bound = LayeredTargets(layer_ptr_cpu, nodes, children, work0, work1, trace, cost, delta, head_v, head_t,
                               head_c, sigma_v, sigma_t, sigma_c, action_p, action_a, conversion, work_cap, head_cap,
                               width, n_replica, input_count, output_count, action_partition_count, p_train,
                               max_width, lambda_, sampled, branched)
        _BINDINGS[key] = bound
        while len(_BINDINGS) > _MAX_BINDINGS:
            _BINDINGS.popitem(last=False)
    else:
        _BINDINGS.move_to_end(key)
    failure = torch.empty(int(n_replica), dtype=torch.int32, device=bound.device)
    return bound.launch(failure_out=failure)


_DATA_PTR = torch.Tensor.data_ptr
_MAX_BINDINGS = 8
_BINDINGS: "OrderedDict[tuple, LayeredTargets]" = OrderedDict()


def clear_bindings() -> None:
    """Drop the cached bindings (they keep their arena tensors alive)."""

    _BINDINGS.clear()


class _Extension:
    """Module-like handle with the reference extension's one entry point."""

    run_layers = staticmethod(run_layers)


def layered_target_cuda() -> _Extension:
    """pbg/core/cuda_layer.py:13: the layer operator, here from the prebuilt libpbgb200.so."""

    if not torch.cuda.is_available():
        raise NativeError("layered targets require CUDA")
    return _Extension()


__all__ = ["BARRIER_TIMEOUT", "INT32_MAX", "LayeredTargets", "TargetError", "clear_bindings", "conversion_table",
           "layered_target_cuda", "run_layers", "synthetic_tree_plan"]


def synthetic_tree_plan(lanes: int, depth: int, branching: int, p_train: int, width: int, *, device,
                        sampled: bool = False, branched: bool = True, lam: float = 0.5, seed: int = 0):
    """A seeded full ``branching``-ary forest (one tree of ``depth`` layers per lane) as run_layers arguments.

    One output and one input partition of ``width`` components.  Work rows are
    double-buffered the way the reference's layer plan lays them out: layer l
    writes arena (l+1)&1 at rows [0, nodes in the layer), the leaves sit in
    arena 0 and are overwritten by layer 1.  Owners follow the player clock
    (layer l is owned by seat l % p_train).  Returns (args, info): ``args`` is
    the positional argument tuple of ``run_layers`` / ``LayeredTargets`` with
    device tensors, ``info`` holds counts and the algorithmic bytes of the pass.
    """

    import numpy as np

    rng = np.random.default_rng(seed)
    b, D, P, W, R = int(branching), int(depth), int(p_train), int(width), int(lanes)
    per_layer = [b ** (D - 1 - layer) for layer in range(D)]
    nodes_per_lane = sum(per_layer)
    cap = b ** D
    cols = {k: [] for k in NODE_COLUMNS}
    src_row, edges_per_node = [], b
    sigma_base = np.cumsum([0] + per_layer)  # per lane: nodes of earlier layers
    layer_ptr = [0]
    for layer, n in enumerate(per_layer):
        lane = np.repeat(np.arange(R), n)
        i = np.tile(np.arange(n), R)
        count = R * n
        cols["replica"].append(lane)
        cols["child_begin"].append(np.zeros(count, np.int64))  # filled below
        cols["child_count"].append(np.full(count, b))
        cols["destination_row"].append(i)
        cols["input_type"].append(np.zeros(count, np.int64))
        cols["output_type"].append(np.zeros(count, np.int64))
        cols["owner_slot"].append(np.full(count, layer % P))
        cols["nominal_degree"].append(np.full(count, b))
        cols["target_degree"].append(np.full(count, b))
        rows = sigma_base[layer] + i
        cols["sigma_head_row"].append(rows)
        cols["sigma_target_row"].append(rows)
        cols["action_begin"].append(rows * b)
        child = (i[:, None] * b + np.arange(b)[None, :]).reshape(-1)
        # layer 0 reads leaves (arena 0); layer l reads layer l-1's rows in arena l&1
        arena = 0 if layer == 0 else layer & 1
        src_row.append(child if arena == 0 else -child - 1)
        layer_ptr.append(layer_ptr[-1] + count)
    node_cols = [np.concatenate(cols[k]).astype(np.int32) for k in NODE_COLUMNS]
    total = int(layer_ptr[-1])
    node_cols[1] = (np.arange(total, dtype=np.int64) * b).astype(np.int32)
    edges = total * b
    children = [np.concatenate(src_row).astype(np.int32), np.zeros(edges, np.int32), np.ones(edges, np.int32),
                rng.uniform(0.5, 1.0, edges).astype(np.float32)]

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device)

    mass = rng.uniform(0.05, 1.0, (R, cap, 2, P, W)).astype(np.float32)
    work0 = [t(mass if not sampled else rng.uniform(-1, 1, mass.shape).astype(np.float32))]
    work1 = [t(mass * rng.uniform(-1, 1, mass.shape).astype(np.float32))] if not sampled else [
        torch.empty(0, device=device)]
    empty = torch.empty(0, device=device)
    trace = [t(rng.uniform(0, 1, (R, cap, 2, P)).astype(np.float32))] if branched else [empty]
    cost = [t(rng.uniform(0, 1, (R, cap, 2)).astype(np.float32))] if branched else [empty]
    delta = [t(rng.uniform(-0.1, 0.1, (R, cap, 2)).astype(np.float32))] if branched else [empty]
    head_v = [t(rng.uniform(-1, 1, (R, nodes_per_lane, W)).astype(np.float32))]
    head_t = [t(rng.uniform(0, 1, (R, nodes_per_lane)).astype(np.float32))] if branched else [empty]
    head_c = [t(rng.uniform(0, 1, (R, nodes_per_lane)).astype(np.float32))] if branched else [empty]
    sigma_v = list(torch.zeros((R, nodes_per_lane, W), device=device).unbind(0))
    sigma_t = list(torch.zeros((R, nodes_per_lane), device=device).unbind(0)) if branched else [empty] * R
    sigma_c = list(torch.zeros((R, nodes_per_lane), device=device).unbind(0)) if branched else [empty] * R
    action_a = list(torch.zeros((R, nodes_per_lane * b, W), device=device).unbind(0))
    action_p = list(torch.zeros((R, nodes_per_lane * b, W), device=device).unbind(0)) if not sampled else [empty] * R
    conversion = torch.arange(W, dtype=torch.int32, device=device)
    args = (torch.tensor(layer_ptr, dtype=torch.int32), [t(c) for c in node_cols], [t(c) for c in children],
            work0, work1, trace, cost, delta, head_v, head_t, head_c, sigma_v, sigma_t, sigma_c, action_p, action_a,
            conversion, [cap], [nodes_per_lane], [W], R, 1, 1, 1, P, W, lam, sampled, branched)
    # algorithmic bytes per node: node record, edges, children's work (and trace/cost/delta) read once,
    # the head row, the parent's work row, sigma and per-action targets written once
    channels = 1 if sampled else 2
    read = 12 * 4 + b * 16 + b * P * W * channels * 4 + W * 4
    write = P * W * channels * 4 + W * 4 + b * W * channels * 4
    if branched:
        read += b * (P + 2) * 4 + 2 * 4
        write += (P + 2) * 4 + 2 * 4
    info = {"lanes": R, "depth": D, "branching": b, "p_train": P, "width": W, "nodes": total, "edges": edges,
            "bytes_per_node": read + write, "algorithmic_bytes": total * (read + write),
            "estimator": "sampled" if sampled else "rao_blackwell", "rollout": "branched" if branched else "sequential"}
    return args, info
