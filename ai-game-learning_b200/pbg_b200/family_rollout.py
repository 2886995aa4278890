"""Family-scheduled rollout with the policy network in the loop.

The reference's rollout (pbg/core/rollout.py:1536-1930 with the queued poker
hooks, hooks.py:1489-2010) groups the live hands of a step into model families
by input partition ("pre" for preflop hands, "post_L" for postflop hands with
L live seats), encodes each family's retained rows (public state, log reach,
public history and, for multiway postflop families, the sealed folded
statistics), evaluates the model on them, and then samples and transitions
every hand.  ``FamilyRollout.step`` does the same on this build's pieces:
``PokerStateMachine.direct_model_input`` (model-input kernel),
``folded_statistics`` + ``pack_folded_statistics`` (folded-statistics kernel),
``QueuedPokerModel.rollout_operation`` (the tensor-core networks), and the
fused ``RolloutStep.step`` / ``reach_update`` kernels, which read each hand's
raw policy rows from one [B, H] buffer (class rows first for preflop hands).

The family codes stay on the device: a stable sort groups the live hands by
family, and the only host read of a step is the per-family count vector
(P + 2 integers), which sizes the model calls as the reference's family
scheduler's sizes do.  The [B, H] raw buffers are allocated once per arena,
and each family is evaluated in chunks of at most ``max_rows`` decisions so
that a postflop call (thousands of tokens per decision) stays within memory
at any batch size.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .folded import folded_statistics, pack_folded_statistics
from .poker import CHECK_CALL, FOLDED, HISTORY_FIELDS, RAISE_OFFSET, STATE_FIELDS, PokerHistory, PokerState
from .queued_model import QueuedPokerModel
from .rollout import RolloutArena, RolloutStep

RAW_FIELDS = ("type_logits", "omega", "mu", "s", "iota")


def tight_folder_mask(history: PokerHistory, status: Tensor) -> Tensor:
    """hooks.py:1609-1620: folded seats that acted voluntarily before folding (instant preflop folds
    are loose)."""

    tight = torch.zeros_like(status, dtype=torch.bool)
    for seat in range(status.shape[1]):
        owned = history.mask & history.actor.eq(seat)
        invested = owned & ((history.action.eq(CHECK_CALL) & history.amount.gt(0)) | history.action.ge(RAISE_OFFSET))
        tight[:, seat] = status[:, seat].eq(FOLDED) & invested.any(-1)
    return tight


class FamilyRollout:
    """Drive a rollout arena with a ``QueuedPokerModel`` evaluated per input family."""

    def __init__(self, model: QueuedPokerModel, *, seed: int, iteration: int,
                 max_rows: dict | None = None) -> None:
        self.model = model
        self.geometry = model.geometry
        self.stepper = RolloutStep(self.geometry, seed=seed, iteration=iteration, with_history=True)
        self.machine = self.stepper.machine
        self.families: dict[str, int] = {}
        self.max_rows = {"pre": 8192, "post": 1024, **(max_rows or {})}
        self._raw: dict | None = None
        self._raw_key = None

    def _raw_buffers(self, rows: int, device) -> dict:
        """[B, H] raw-policy buffers, allocated once per arena size (a neutral policy in every slot)."""

        key = (rows, str(device))
        if self._raw_key != key:
            H, M = self.geometry.private_hands, self.model.cfg.m_raise
            self._raw = {"type_logits": torch.zeros((rows, H, 3), device=device),
                         "omega": torch.full((rows, H, M), 1.0 / M, device=device),
                         "mu": torch.full((rows, H, M), 0.5, device=device),
                         "s": torch.ones((rows, H, M), device=device),
                         "iota": torch.full((rows, H), 0.5, device=device)}
            self._raw_key = key
        return self._raw

    def roots(self, rows: int, *, device, retry_epoch: int = 0, logical_base: int = 0,
              lane: int = 0) -> tuple[RolloutArena, Tensor]:
        """Fresh roots and their public log reach (every private hand equally likely: 0)."""

        arena = self.stepper.roots(rows, device=device, retry_epoch=retry_epoch, logical_base=logical_base, lane=lane)
        g = self.geometry
        return arena, torch.zeros((rows, g.players, g.private_hands), dtype=torch.float32, device=arena.state.device)

    def _family_rows(self, arena: RolloutArena, kind: str, rows: Tensor, log_reach: Tensor) -> Tensor:
        """The retained model-input rows of one family (hooks.py:531-612, 1968-2006)."""

        g = self.geometry
        state = PokerState(*(getattr(arena.state, n).index_select(0, rows).contiguous() for n in STATE_FIELDS))
        history = PokerHistory(*(getattr(arena.history, n).index_select(0, rows).contiguous() for n in HISTORY_FIELDS))
        reach = log_reach.index_select(0, rows).contiguous()
        model_input = self.machine.direct_model_input(kind, state, reach, history)
        if kind != "pre" and g.folded_summary_width:
            summary = folded_statistics(
                g, board_cards=state.board_cards, range_weights=torch.exp(reach).masked_fill(~torch.isfinite(reach), 0.0),
                status=state.status, combo_cards=self.model.combo_cards.to(torch.int32), beta_rank=g.deck_cards,
                line_dim=0, tight_mask=tight_folder_mask(history, state.status))
            model_input[:, g.postflop_base_model_input_width:] = pack_folded_statistics(g, summary)
        return model_input, state

    def step(self, arena: RolloutArena, log_reach: Tensor) -> int:
        """One player decision for every live hand, every family's raw policy from the model.
        Returns the number of decisions taken (0 when every hand is terminal)."""

        g = self.geometry
        state = arena.state
        # family of each hand (hooks.py:456-462, pbg_input_type: pre 0, post_A A - 1), -1 once terminal
        code = torch.where(state.terminal, -1, self.machine.input_type(state))
        counts = torch.bincount(code + 1, minlength=g.players + 1).cpu().tolist()  # the step's one host read
        decisions = sum(counts[1:])
        if decisions == 0:
            return 0
        raw = self._raw_buffers(arena.rows, state.device)
        order = torch.sort(code, stable=True).indices  # terminal hands first, then each family in index order
        start = counts[0]
        for value, count in enumerate(counts[1:]):
            if count == 0:
                continue
            kind = "pre" if value == 0 else f"post_{value + 1}"
            chunk = self.max_rows["pre" if value == 0 else "post"]
            family = order[start:start + count]
            start += count
            for lo in range(0, count, chunk):
                rows = family[lo:lo + chunk]
                model_input, sub = self._family_rows(arena, kind, rows, log_reach)
                evaluation = self.model.rollout_operation(kind, model_input, sub.combo_ids, sub.to_act.to(torch.int64))
                for name in RAW_FIELDS:
                    field = evaluation.policy_raw[name]
                    raw[name][rows, : field.shape[1]] = field.float()
            self.families[kind] = self.families.get(kind, 0) + count
        self.stepper.step(arena, raw)
        self.stepper.reach_update(arena, raw, log_reach)
        return decisions


__all__ = ["FamilyRollout", "tight_folder_mask"]
