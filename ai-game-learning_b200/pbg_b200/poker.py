"""NLHE geometry, public state and state machine on the device.

Mirrors pbg/games/poker/queued/hooks.py:72-1216 (NLHEGeometry, PokerState,
PokerHistory, PokerStateMachine) with every transition executed by
libpbgb200's sm_100a kernels.  Tensor dtypes and shapes are the
reference's, so states move between the two without conversion.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, fields, replace
from types import MappingProxyType

import torch
from torch import Tensor

from . import _native as N
from ._native import call, ptr, stream

PAD_CARD = 255
LIVE = 0
FOLDED = 1
ALL_IN = 2
FOLD = 0
CHECK_CALL = 1
RAISE_OFFSET = 2


class QueuedPokerError(RuntimeError):
    """The queued poker state or evaluator contract was violated."""


def max_public_history_tokens(n_players: int, stack_bb: float) -> int:
    """pbg/games/poker/model/capacity.py:12-25."""

    return math.ceil(stack_bb * n_players + 3 * n_players - stack_bb + 1) + 3


@dataclass(frozen=True)
class NLHEGeometry:
    """hooks.py:72-192."""

    players: int
    stack_bb: float
    rank_count: int

    def __post_init__(self) -> None:
        if isinstance(self.players, bool) or not isinstance(self.players, int) or not 2 <= self.players <= 6:
            raise ValueError("players must be an integer in [2,6]")
        if (isinstance(self.stack_bb, bool) or not isinstance(self.stack_bb, (int, float))
                or not math.isfinite(self.stack_bb) or not 8 <= self.stack_bb <= 128
                or not math.isclose(self.stack_bb * 2, round(self.stack_bb * 2))):
            raise ValueError("stack_bb must be a half-integer in [8,128]")
        if isinstance(self.rank_count, bool) or not isinstance(self.rank_count, int) or not 4 <= self.rank_count <= 13:
            raise ValueError("rank_count must be an integer in [4,13]")
        if 2 * self.players + 5 >= self.deck_cards:
            raise ValueError("NLHE geometry must satisfy 2P+5<4R")

    @property
    def deck_cards(self) -> int:
        return 4 * self.rank_count

    @property
    def first_card(self) -> int:
        return 52 - self.deck_cards

    @property
    def private_hands(self) -> int:
        return self.deck_cards * (self.deck_cards - 1) // 2

    @property
    def private_classes(self) -> int:
        return self.rank_count ** 2

    @property
    def stack_ticks(self) -> int:
        return round(self.stack_bb * 2)

    @property
    def events(self) -> int:
        return self.stack_ticks + RAISE_OFFSET

    @property
    def history_tokens(self) -> int:
        return max_public_history_tokens(self.players, self.stack_bb)

    @property
    def c(self) -> N.Geometry:
        return N.Geometry(self.players, self.stack_ticks, self.rank_count)

    @property
    def player_node_bound(self) -> int:
        return math.ceil(self.stack_bb * self.players + 3 * self.players - self.stack_bb + 1)

    def model_private_width(self, input_type: str) -> int:
        """hooks.py:164-169."""

        if input_type == "pre":
            return self.private_classes
        if input_type.startswith("post_") and input_type[5:].isdigit():
            return self.private_hands
        raise ValueError(f"unknown poker input partition {input_type!r}")

    @property
    def public_model_input_width(self) -> int:
        return 8 + 10 * self.players

    @property
    def history_model_input_width(self) -> int:
        return 10 * self.history_tokens

    @property
    def preflop_model_input_width(self) -> int:
        return self.public_model_input_width + self.players * self.private_classes + self.history_model_input_width

    @property
    def postflop_base_model_input_width(self) -> int:
        return self.public_model_input_width + self.players * self.private_hands + self.history_model_input_width

    @property
    def folded_summary_width(self) -> int:
        """hooks.py:171-185: Lambda_B [H], full-rank beta eigenpairs [C + C*C], folder log masses [P],
        card masses [P*C], tight scalar and validity flag; none heads-up (a fold is terminal)."""

        if self.players == 2:
            return 0
        cards = self.deck_cards
        return self.private_hands + cards + cards * cards + self.players + self.players * cards + 2

    @property
    def postflop_model_input_width(self) -> int:
        return self.postflop_base_model_input_width + self.folded_summary_width

    def model_input_width(self, input_type: str) -> int:
        """hooks.py:157-162."""

        if input_type == "pre":
            return self.preflop_model_input_width
        if input_type.startswith("post_") and input_type[5:].isdigit():
            return self.postflop_model_input_width
        raise ValueError(f"unknown poker input partition {input_type!r}")

    def combo_id(self, first: Tensor, second: Tensor) -> Tensor:
        low = torch.minimum(first, second).to(torch.int64) - self.first_card
        high = torch.maximum(first, second).to(torch.int64) - self.first_card
        return (low * (2 * self.deck_cards - low - 1) // 2 + high - low - 1).to(torch.int32)


STATE_FIELDS = ("board_cards", "combo_ids", "button", "street", "to_act", "stacks", "committed",
                "committed_street", "status", "current_bet", "last_full_raise", "pending", "can_raise",
                "terminal")


@dataclass(frozen=True)
class PokerState:
    """hooks.py:250-326: device-resident public state of independent hands."""

    board_cards: Tensor
    combo_ids: Tensor
    button: Tensor
    street: Tensor
    to_act: Tensor
    stacks: Tensor
    committed: Tensor
    committed_street: Tensor
    status: Tensor
    current_bet: Tensor
    last_full_raise: Tensor
    pending: Tensor
    can_raise: Tensor
    terminal: Tensor

    @property
    def rows(self) -> int:
        return self.board_cards.shape[0]

    @property
    def device(self) -> torch.device:
        return self.board_cards.device

    @classmethod
    def empty(cls, rows: int, players: int, device) -> "PokerState":
        f = lambda shape, dt: torch.zeros(shape, dtype=dt, device=device)
        return cls(f((rows, 5), torch.uint8), f((rows, players), torch.int32), f(rows, torch.int32),
                   f(rows, torch.int32), f(rows, torch.int32), f((rows, players), torch.float32),
                   f((rows, players), torch.float32), f((rows, players), torch.float32),
                   f((rows, players), torch.int8), f(rows, torch.float32), f(rows, torch.float32),
                   f((rows, players), torch.bool), f((rows, players), torch.bool), f(rows, torch.bool))

    def clone(self) -> "PokerState":
        return PokerState(*(getattr(self, n).clone() for n in STATE_FIELDS))

    def validate(self, geometry: NLHEGeometry) -> None:
        batch, players = self.rows, geometry.players
        dtypes = {"board_cards": (torch.uint8, (batch, 5)), "combo_ids": (torch.int32, (batch, players)),
                  "button": (torch.int32, (batch,)), "street": (torch.int32, (batch,)),
                  "to_act": (torch.int32, (batch,)), "stacks": (torch.float32, (batch, players)),
                  "committed": (torch.float32, (batch, players)),
                  "committed_street": (torch.float32, (batch, players)),
                  "status": (torch.int8, (batch, players)), "current_bet": (torch.float32, (batch,)),
                  "last_full_raise": (torch.float32, (batch,)), "pending": (torch.bool, (batch, players)),
                  "can_raise": (torch.bool, (batch, players)), "terminal": (torch.bool, (batch,))}
        for name, (dtype, shape) in dtypes.items():
            value = getattr(self, name)
            if value.device != self.device or not value.is_cuda or value.dtype != dtype or tuple(value.shape) != shape \
                    or not value.is_contiguous():
                raise QueuedPokerError(f"{name} must be contiguous CUDA {dtype} with shape {shape}")

    def c(self) -> N.State:
        return N.State(*(ptr(getattr(self, n)) for n in STATE_FIELDS))


HISTORY_FIELDS = ("actor", "street", "action", "amount", "pot_before", "call_amount", "current_bet",
                  "min_raise_to", "max_raise_to", "mask")


@dataclass(frozen=True)
class PokerHistory:
    """hooks.py:329-339."""

    actor: Tensor
    street: Tensor
    action: Tensor
    amount: Tensor
    pot_before: Tensor
    call_amount: Tensor
    current_bet: Tensor
    min_raise_to: Tensor
    max_raise_to: Tensor
    mask: Tensor

    def clone(self) -> "PokerHistory":
        return PokerHistory(*(getattr(self, n).clone() for n in HISTORY_FIELDS))

    def c(self, length: Tensor | None = None) -> N.History:
        """ABI view; `length` ([B] int32 tokens used) lets appends skip counting the mask."""

        return N.History(*(ptr(getattr(self, n)) for n in HISTORY_FIELDS), self.mask.shape[1], ptr(length))


@dataclass(frozen=True)
class PokerLegality:
    """policy.py:30-56: fixed-width public legal event rows."""

    event_ids: Tensor
    mask: Tensor

    @property
    def raise_ticks(self) -> int:
        return self.event_ids.shape[1] - RAISE_OFFSET


class PokerStateMachine:
    """hooks.py:351-1216 on libpbgb200 kernels (in-place on cloned states)."""

    def __init__(self, geometry: NLHEGeometry) -> None:
        self.geometry = geometry

    def _leaf_tensors(self, rows, device):
        P = self.geometry.players
        return {
            "leaf_public_state": torch.empty((rows, 5), dtype=torch.uint8, device=device),
            "leaf_private_profile": torch.empty((rows, P), dtype=torch.int32, device=device),
            "stratum_level": torch.empty((rows, P), dtype=torch.int32, device=device),
            "payoff_baseline": torch.empty((rows, P), dtype=torch.float32, device=device),
            "stratum_amount": torch.empty((rows, P), dtype=torch.float32, device=device),
        }

    def initial_roots(self, root_count: int, *, seed: int, iteration: int, retry_epoch: int,
                      logical_base: int = 0, buttons: Tensor | None = None, lane: int = 0,
                      device) -> PokerState:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("queued poker roots require CUDA")
        if root_count <= 0:
            raise ValueError("root_count must be positive")
        state = PokerState.empty(root_count, self.geometry.players, device)
        b = None
        if buttons is not None:
            if buttons.shape != (root_count,) or bool(((buttons < 0) | (buttons >= self.geometry.players)).any()):
                raise ValueError("explicit root buttons must be accelerator integers in [0,P)")
            b = buttons.to(device=device, dtype=torch.int32).contiguous()
        call("pbg_initial_roots", self.geometry.c, root_count, int(seed), int(iteration), int(retry_epoch),
             int(logical_base), int(lane), ptr(b), state.c(), stream(device))
        return state

    def input_type(self, state: PokerState) -> Tensor:
        out = torch.empty(state.rows, dtype=torch.int32, device=state.device)
        call("pbg_input_type", self.geometry.c, state.rows, state.c(), ptr(out), stream(state.device))
        return out

    def legality(self, state: PokerState) -> PokerLegality:
        """hooks.py:464-510, through the ``pbg_b200::legality`` operator (traceable by torch.compile)."""

        from .ops import legality as legality_op

        E = self.geometry.events
        g = self.geometry
        mask = legality_op(*(getattr(state, n) for n in STATE_FIELDS), g.players, g.stack_ticks, g.rank_count)
        ids = torch.arange(E, dtype=torch.int32, device=state.device)[None].expand(state.rows, -1).contiguous()
        return PokerLegality(ids, mask)

    def step_player(self, state: PokerState, action: Tensor) -> PokerState:
        if action.shape != (state.rows,):
            raise QueuedPokerError("player action must have shape [B]")
        out = state.clone()
        a = action.to(torch.int32).contiguous()
        call("pbg_step_player", self.geometry.c, out.rows, out.c(), ptr(a), stream(out.device))
        return out

    def needs_chance(self, state: PokerState) -> Tensor:
        out = torch.empty(state.rows, dtype=torch.bool, device=state.device)
        call("pbg_needs_chance", self.geometry.c, state.rows, state.c(), ptr(out), stream(state.device))
        return out

    def deal_next_street(self, state: PokerState, logical_key: Tensor, *, active: Tensor | None = None) -> PokerState:
        if logical_key.shape != (state.rows, self.geometry.deck_cards):
            raise QueuedPokerError("chance keys must be [B,D]")
        out = state.clone()
        call("pbg_deal_next_street", self.geometry.c, out.rows, out.c(), ptr(logical_key.contiguous()),
             ptr(None if active is None else active.contiguous()), stream(out.device))
        return out

    def deal_next_street_keyed(self, state: PokerState, *, seed: int, iteration: int, root: Tensor, path: Tensor,
                               draw: int, retry_epoch, lane=0, active: Tensor | None = None) -> PokerState:
        if root.shape != (state.rows,) or path.shape != root.shape:
            raise QueuedPokerError("chance root/path addresses must be CUDA [B]")
        out = state.clone()
        full = lambda v: (v.to(torch.int64) if isinstance(v, Tensor) else torch.full_like(root, int(v),
                                                                                        dtype=torch.int64)).contiguous()
        call("pbg_deal_next_street_keyed", self.geometry.c, out.rows, out.c(), int(seed), int(iteration),
             ptr(root.to(torch.int64).contiguous()), ptr(path.to(torch.int64).contiguous()), int(draw),
             ptr(full(retry_epoch)), ptr(full(lane)), ptr(None if active is None else active.contiguous()),
             stream(out.device))
        return out

    def empty_history(self, rows: int, device) -> PokerHistory:
        tokens = self.geometry.history_tokens
        integer = torch.full((rows, tokens), -1, dtype=torch.int64, device=device)
        numeric = torch.zeros((rows, tokens), dtype=torch.float32, device=device)
        return PokerHistory(integer.clone(), integer.clone(), integer.clone(), *(numeric.clone() for _ in range(6)),
                            torch.zeros((rows, tokens), dtype=torch.bool, device=device))

    def append_player_history(self, state: PokerState, action: Tensor, history: PokerHistory) -> PokerHistory:
        out = history.clone()
        call("pbg_append_player_history", self.geometry.c, state.rows, state.c(),
             ptr(action.to(torch.int32).contiguous()), out.c(), stream(state.device))
        return out

    def append_chance_history(self, state: PokerState, active: Tensor, history: PokerHistory) -> PokerHistory:
        out = history.clone()
        call("pbg_append_chance_history", self.geometry.c, state.rows, state.c(), ptr(active.contiguous()),
             out.c(), stream(state.device))
        return out

    def sampled_leaf(self, state: PokerState):
        leaf = self._leaf_tensors(state.rows, state.device)
        call("pbg_sampled_leaf", self.geometry.c, state.rows, state.c(),
             N.Leaf(*(ptr(v) for v in leaf.values())), stream(state.device))
        return MappingProxyType(leaf)

    def rb_leaf(self, state: PokerState, log_reach: Tensor, *, seed: Tensor, selected_player: Tensor | None = None):
        """hooks.py:1218-1258: the contract-v2 completion inputs of Rao-Blackwell leaves.

        The public pre-terminal board stays as it is (an early fold is not padded with dealt
        cards, which would move it between the pre- and post-flop outputs); the stratum fields are
        the sampled settlement's with the hand forced terminal; each seat's range weights are
        exp(log_reach - its largest finite reach), non-finite reaches weighing 0."""

        g = self.geometry
        if (log_reach.shape != (state.rows, g.players, g.private_hands) or log_reach.dtype != torch.float32
                or log_reach.device != state.device):
            raise QueuedPokerError("RB leaf reaches must be CUDA FP32 [B,P,H]")
        sampled = self.sampled_leaf(replace(state, terminal=torch.ones_like(state.terminal)))
        finite = torch.isfinite(log_reach)
        top = torch.where(finite, log_reach, -torch.inf).amax(-1, keepdim=True)
        top = torch.where(torch.isfinite(top), top, 0.0)
        weights = torch.where(finite, torch.exp(log_reach - top), 0.0)
        leaf = {
            "leaf_public_state": state.board_cards.contiguous(),
            "stratum_level": sampled["stratum_level"],
            "payoff_baseline": sampled["payoff_baseline"],
            "stratum_amount": sampled["stratum_amount"],
            "range_weights": weights.contiguous(),
            "seed": seed.to(dtype=torch.int64, device=state.device).contiguous(),
        }
        if selected_player is not None:
            leaf["trained_actor"] = selected_player.to(dtype=torch.int32, device=state.device).contiguous()
        return MappingProxyType(leaf)

    def model_input_width(self, input_type: str) -> int:
        """hooks.py:138-169: retained row width of a partition."""

        return self.geometry.model_input_width(input_type)

    def direct_model_input(self, input_type: str, state: PokerState, log_reach: Tensor | None = None,
                           history: PokerHistory | None = None) -> Tensor:
        """hooks.py:531-612: the retained public, reach and history model row."""

        width = self.model_input_width(input_type)
        pre = input_type == "pre"
        if log_reach is not None and log_reach.shape != (state.rows, self.geometry.players,
                                                          self.geometry.private_hands):
            raise QueuedPokerError("device model input takes the exact [B,P,H] reach")
        out = torch.empty((state.rows, width), dtype=torch.float32, device=state.device)
        hist = history.c() if history is not None else N.History(*([None] * 10), self.geometry.history_tokens, None)
        call("pbg_direct_model_input", self.geometry.c, state.rows, state.c(), 0 if pre else 1,
             ptr(None if log_reach is None else log_reach.float().contiguous()), hist, ptr(out), width,
             stream(state.device))
        return out

    def state_from_model_input(self, input_type: str, model_input: Tensor, combo_ids: Tensor) -> PokerState:
        """hooks.py:812-881: the public transition state recovered from a retained model-input row
        (the layout direct_model_input writes), with the given private combos."""

        g = self.geometry
        players = g.players
        if (not model_input.is_cuda or model_input.dtype not in (torch.float32, torch.float16, torch.bfloat16)
                or model_input.ndim != 2 or model_input.shape[1] != g.model_input_width(input_type)
                or combo_ids.shape != (model_input.shape[0], players) or combo_ids.dtype != torch.int32
                or combo_ids.device != model_input.device):
            raise QueuedPokerError("retained model input cannot reconstruct poker state")
        value = model_input.float()
        widths = (1, 5, players, players, players, players, players, 3 * players, players, 1, 1, players)
        parts = torch.split(value[:, : sum(widths)], widths, dim=1)
        scale = float(g.stack_bb)
        board = torch.where(parts[1] < 0, torch.full_like(parts[1], PAD_CARD),
                            torch.round(parts[1] * max(1, g.deck_cards - 1) + g.first_card)).to(torch.uint8)
        state = PokerState(
            board.contiguous(), combo_ids.contiguous(), parts[3].argmax(-1).to(torch.int32),
            torch.round(parts[0][:, 0] * 3).to(torch.int32), parts[2].argmax(-1).to(torch.int32),
            (parts[4] * scale).contiguous(), (parts[5] * scale).contiguous(), (parts[6] * scale).contiguous(),
            parts[7].reshape(-1, players, 3).argmax(-1).to(torch.int8), (parts[9][:, 0] * scale).contiguous(),
            (parts[10][:, 0] * scale).contiguous(), parts[8].gt(0.5).contiguous(), parts[11].gt(0.5).contiguous(),
            torch.zeros(model_input.shape[0], dtype=torch.bool, device=model_input.device))
        state.validate(g)
        return state

    def model_context(self, input_type: str, model_input: Tensor) -> tuple[Tensor, PokerHistory]:
        """hooks.py:665-699: the retained log reach [B, P, K or H] and public history of a row."""

        g = self.geometry
        players, width, tokens = g.players, g.model_private_width(input_type), g.history_tokens
        offset = 8 + 10 * players
        reach = model_input[:, offset: offset + players * width].float()
        offset += players * width
        columns = [model_input[:, offset + i * tokens: offset + (i + 1) * tokens] for i in range(10)]
        offset += 10 * tokens
        base = g.preflop_model_input_width if input_type == "pre" else g.postflop_base_model_input_width
        if offset != base or model_input.shape[1] != g.model_input_width(input_type):
            raise QueuedPokerError("retained model context layout is not exact")
        history = PokerHistory(*(columns[i].round().to(torch.int64) for i in range(3)),
                               *(columns[i].float() for i in range(3, 9)), columns[9].gt(0.5))
        return reach.reshape(-1, players, width), history

    def expand_preflop_reach(self, compact: Tensor) -> Tensor:
        """hooks.py:650-655: class-wide log reach spread to every combo of its class."""

        if compact.shape[-1] != self.geometry.private_classes:
            raise QueuedPokerError("preflop reach is not class-wide")
        classes = self._combo_class(compact.device)
        counts = torch.bincount(classes, minlength=self.geometry.private_classes).to(torch.float32)
        return compact.index_select(-1, classes) - counts.log().index_select(0, classes)

    def exact_model_context(self, input_type: str, model_input: Tensor) -> tuple[Tensor, PokerHistory]:
        """hooks.py:701-706."""

        reach, history = self.model_context(input_type, model_input)
        return (self.expand_preflop_reach(reach) if input_type == "pre" else reach), history

    def combo_cards(self, combo_ids: Tensor) -> Tensor:
        ids = combo_ids.to(torch.int32).contiguous()
        out = torch.empty(ids.shape + (2,), dtype=torch.int64, device=ids.device)
        call("pbg_combo_cards", self.geometry.c, ids.numel(), ptr(ids), ptr(out), stream(ids.device))
        return out

    def _combo_class(self, device) -> Tensor:
        out = torch.empty(self.geometry.private_hands, dtype=torch.int32, device=device)
        call("pbg_combo_class", self.geometry.c, ptr(out), stream(torch.device(device)))
        return out.to(torch.int64)
