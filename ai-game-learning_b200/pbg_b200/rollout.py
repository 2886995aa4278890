"""Fused sampled rollout step over a device arena of independent hands.

One ``RolloutStep.step`` call does, for every non-terminal hand, what the
reference spreads over a family-scheduled transaction
(pbg/core/rollout.py:1536-1930 with hooks.py:1489-1870): the ACTION key at
(root, path, draw 0), sampling from the composite policy at the owner's
private row, the history append, step_player, three keyed chance
generations, the sampled-leaf payload of hands that end, and the child
path.  ``reach_update`` then adds the selected action's log policy of every
private hand to the actor's reach row and masks board conflicts
(hooks.py:1641-1703).

Because keys are addressed by (root, path), results do not depend on how
hands are batched or ordered, exactly as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from ._native import call, ptr, stream
from .poker import NLHEGeometry, PokerHistory, PokerState, PokerStateMachine
from .policy import policy_struct


@dataclass
class RolloutArena:
    """Device-resident columns of B hands (SoA)."""

    state: PokerState
    history: PokerHistory
    root_path: Tensor      # [B,2] int64 (root, path)
    lane: Tensor           # [B] int64
    retry_epoch: Tensor    # [B] int64
    action: Tensor         # [B] int32 (last step)
    selected_log: Tensor   # [B] fp32
    decision: Tensor       # [B,4] int32
    new_leaf: Tensor       # [B] bool
    leaf: dict             # sampled_leaf columns
    history_length: Tensor  # [B] int32 tokens used (kept by the kernel)
    worklist: Tensor | None = None  # [B+1] int32: the live hands of the current step (count first)

    @property
    def rows(self) -> int:
        return self.state.rows


class RolloutStep:
    def __init__(self, geometry: NLHEGeometry, *, seed: int, iteration: int, with_history: bool = True,
                 work_list: bool = False) -> None:
        self.geometry = geometry
        # work_list: list the live hands first and step them in dense warps (pbg_rollout_step_listed).
        # Same results; on the HU 100bb rollout it is slower than one thread per row (the extra pass
        # and the gathered state cost more than the idle lanes of finished hands).
        self.work_list = work_list
        self.machine = PokerStateMachine(geometry)
        self.seed = int(seed)
        self.iteration = int(iteration)
        self.with_history = with_history

    def roots(self, rows: int, *, device, retry_epoch: int = 0, logical_base: int = 0, lane: int = 0) -> RolloutArena:
        device = torch.device(device)
        state = self.machine.initial_roots(rows, seed=self.seed, iteration=self.iteration, retry_epoch=retry_epoch,
                                           logical_base=logical_base, lane=lane, device=device)
        history = self.machine.empty_history(rows if self.with_history else 0, device)
        root = torch.arange(logical_base, logical_base + rows, dtype=torch.int64, device=device)
        root_path = torch.stack((root, torch.zeros_like(root)), 1).contiguous()
        return RolloutArena(
            state, history, root_path,
            torch.full((rows,), lane, dtype=torch.int64, device=device),
            torch.full((rows,), retry_epoch, dtype=torch.int64, device=device),
            torch.full((rows,), -1, dtype=torch.int32, device=device),
            torch.zeros(rows, dtype=torch.float32, device=device),
            torch.zeros((rows, 4), dtype=torch.int32, device=device),
            torch.zeros(rows, dtype=torch.bool, device=device),
            self.machine._leaf_tensors(rows, device),
            torch.zeros(rows, dtype=torch.int32, device=device),
            torch.zeros(rows + 1, dtype=torch.int32, device=device) if self.work_list else None)

    def step(self, arena: RolloutArena, raw) -> None:
        """Advance every non-terminal hand by one player decision (in place).

        With the arena's work list (``work_list=True``) the live hands are listed first and the step
        runs dense warps over them (``pbg_rollout_step_listed``); the results are the same."""

        pol, keep, rows = policy_struct(raw)
        hist = arena.history.c(arena.history_length) if self.with_history else N.History(*([None] * 10), 0, None)
        leaf = N.Leaf(*(ptr(v) for v in arena.leaf.values()))
        args = (self.geometry.c, arena.rows, arena.state.c(), hist, ptr(arena.root_path), ptr(arena.lane),
                ptr(arena.retry_epoch), self.seed, self.iteration, pol, ptr(arena.action), ptr(arena.selected_log),
                ptr(arena.decision), ptr(arena.new_leaf), leaf)
        if arena.worklist is not None:
            call("pbg_rollout_step_listed", *args, ptr(arena.worklist), stream(arena.state.device))
        else:
            call("pbg_rollout_step", *args, stream(arena.state.device))

    def reach_update(self, arena: RolloutArena, raw, log_reach: Tensor) -> None:
        """hooks.py:1641-1703 for the decision just taken (in place)."""

        pol, keep, rows = policy_struct(raw)
        if log_reach.shape != (arena.rows, self.geometry.players, self.geometry.private_hands):
            raise ValueError("log_reach must be [B,P,H]")
        call("pbg_reach_update", self.geometry.c, arena.rows, arena.state.c(), pol, ptr(arena.action),
             ptr(arena.decision), ptr(log_reach), stream(arena.state.device))
