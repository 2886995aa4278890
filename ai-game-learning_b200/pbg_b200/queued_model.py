"""The queued poker model operation (pbg/games/poker/queued/model.py) on this build's kernels.

``QueuedPokerModel`` is the model entry point of the rollout and the learner:
it takes the retained model-input rows of a partition ("pre", or "post_L" for L
live seats), recovers the public state, the log reach and the public history
from them (``PokerStateMachine.state_from_model_input`` / ``model_context``,
hooks.py:665-881), assembles the encoder inputs the way the reference does
(model.py:191-350: the public batch with legality-derived raise bounds, class
or combo ranges normalised per seat, the board compatibility of every combo,
the live seats and the retained folded summary), and runs the preflop or the
postflop network (``PreflopModel`` / ``PostflopModel``: tcgen05 dense maps,
the tensor-core attention core, LayerNorm and incidence kernels).  It binds the
reference's own ``state_dict`` (``shared.*``, ``pre_encoder.*``,
``post_encoder.*``).  The decoding steps are torch operations on the device;
legality runs on the state-machine kernel.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from types import MappingProxyType

import torch
from torch import Tensor

from .checks import _assert
from .folded import unpack_folded_statistics
from .postflop import PostflopMasks, PostflopModel
from .poker import FOLD, FOLDED, PAD_CARD, NLHEGeometry, PokerHistory, PokerState, PokerStateMachine
from .preflop import PolicyOutput, PreflopConfig, PreflopModel


class PokerModelError(RuntimeError):
    """A partition model violated the queued model operation (model.py:38-39)."""


@dataclass(frozen=True)
class ModelEvaluation:
    """learner.py:324-331: one model result before the canonical policy reduction."""

    policy_raw: MappingProxyType
    value: Tensor
    public_heads: MappingProxyType = field(default_factory=lambda: MappingProxyType({}))


def fold_line_metadata(history: PokerHistory, status: Tensor, *, line_dim: int, stack_bb: float) -> Tensor:
    """model.py:42-89: each folded seat's retained action line at its fold event, [B, P, line_dim]."""

    tokens = history.mask.shape[1]
    players = status.shape[1]
    position = torch.arange(tokens, device=status.device)[None]
    rows = []
    for seat in range(players):
        folder = status[:, seat].eq(FOLDED)
        owned = history.mask & history.actor.eq(seat)
        fold = owned & history.action.eq(FOLD)
        _assert((~folder | fold.any(-1)).all(), "folded seat has no retained fold-line event")
        last = torch.where(fold, position, torch.full_like(position, -1)).max(-1).values
        at = last.clamp_min(0)[:, None]
        through = owned & position.le(last[:, None])
        calls = through & history.action.eq(1)
        raises = through & history.action.eq(2)
        values = (history.street.gather(1, at).squeeze(1).float() / 3.0,
                  through.sum(-1, dtype=torch.float32) / max(tokens, 1),
                  (history.amount * through).sum(-1) / float(stack_bb),
                  calls.sum(-1, dtype=torch.float32),
                  raises.sum(-1, dtype=torch.float32),
                  history.amount.gather(1, at).squeeze(1) / float(stack_bb),
                  history.pot_before.gather(1, at).squeeze(1) / float(stack_bb),
                  history.call_amount.gather(1, at).squeeze(1) / float(stack_bb))
        if line_dim:
            rows.append(torch.stack(tuple(torch.where(folder, v, torch.zeros_like(v)) for v in values[:line_dim]), -1))
        else:
            rows.append(history.amount[:, :0])
    return torch.stack(tuple(rows), 1)


def _split(params: dict, prefix: str) -> dict:
    return {name[len(prefix):]: value for name, value in params.items() if name.startswith(prefix)}


class QueuedPokerModel:
    """model.py:147-452: one shared model routed through the preflop and postflop networks."""

    def __init__(self, geometry: NLHEGeometry, config: PreflopConfig, params: dict[str, Tensor], device) -> None:
        if config.max_players < geometry.players:
            raise PokerModelError("model max_players does not cover all seats")
        self.geometry, self.cfg, self.device = geometry, config, torch.device(device)
        shared = _split(params, "shared.")
        self._shared_names = frozenset(shared)
        self.pre = PreflopModel(config, geometry.rank_count, {**shared, **_split(params, "pre_encoder.")}, device)
        self.post = PostflopModel(config, geometry.rank_count, {**shared, **_split(params, "post_encoder.")}, device)
        self.machine = PokerStateMachine(geometry)
        self.combo_class = self.machine._combo_class(self.device)
        self.combo_cards = self.machine.combo_cards(
            torch.arange(geometry.private_hands, dtype=torch.int32, device=self.device)).to(torch.int64)

    # ------------------------------------------------------------ training
    def enable_training(self):
        """Put both partition networks in training mode over ONE set of parameters: every parameter
        (``shared.*``, ``pre_encoder.*``, ``post_encoder.*``) a leaf view of one flat fp32 master, the
        shared ones the same leaves in both networks.  Returns the ``FlatParameters``."""

        from .model_train import FlatParameters

        def full(prefix: str, name: str) -> str:
            return ("shared." if name in self._shared_names else prefix) + name

        params = {full("pre_encoder.", n): v for n, v in self.pre.p.items()}
        params.update({full("post_encoder.", n): v for n, v in self.post.p.items()})
        flat = FlatParameters(params, self.device)
        self.pre.bind_parameters({n: flat.leaves[full("pre_encoder.", n)] for n in self.pre.p})
        self.post.bind_parameters({n: flat.leaves[full("post_encoder.", n)] for n in self.post.p})
        self.pre.train()
        self.post.train()
        return flat

    def eval(self) -> "QueuedPokerModel":
        """Back to inference mode (the maps' bf16 operands refreshed from the current parameters)."""

        self.pre.train(False)
        self.post.train(False)
        return self

    # ------------------------------------------------------------ input decoding
    def _state(self, input_type: str, model_input: Tensor) -> PokerState:
        combo_ids = torch.zeros((model_input.shape[0], self.geometry.players), dtype=torch.int32,
                                device=model_input.device)
        return self.machine.state_from_model_input(input_type, model_input, combo_ids)

    def _public(self, state: PokerState, history: PokerHistory):
        """model.py:201-273: the encoders' public batch and the board compatibility of every combo."""

        g = self.geometry
        legality = self.machine.legality(state)
        raise_mask = legality.mask[:, 2:]
        raise_ticks = (torch.arange(1, g.stack_ticks + 1, dtype=torch.float32, device=state.device)[None]
                       * 0.5).expand(state.rows, -1)
        lower = raise_ticks.masked_fill(~raise_mask, torch.inf).min(1).values
        upper = raise_ticks.masked_fill(~raise_mask, -torch.inf).max(1).values
        has_raise = raise_mask.any(1)
        lower = torch.where(has_raise, lower, torch.zeros_like(lower))
        upper = torch.where(has_raise, upper, torch.zeros_like(upper))
        actor = state.to_act.to(torch.int64)
        actor_committed = state.committed_street.gather(1, actor[:, None]).squeeze(1)
        board = torch.where(state.board_cards.eq(PAD_CARD), torch.full_like(state.board_cards, -1, dtype=torch.int64),
                            state.board_cards.to(torch.int64))
        public = {
            "street": state.street.to(torch.int64), "board": board, "pot": state.committed.sum(1),
            "stacks": state.stacks, "committed": state.committed, "to_act": actor,
            "legality_summary": torch.stack((legality.mask[:, 0].float(), legality.mask[:, 1].float(),
                                             raise_mask.float().mean(1)), 1),
            "n_ticks": torch.full((state.rows,), g.stack_ticks, dtype=torch.int64, device=state.device),
            "raise_grid_bounds": torch.stack((lower, upper), 1), "status": state.status.to(torch.int64),
            "seat_mask": torch.ones_like(state.status, dtype=torch.bool), "button": state.button.to(torch.int64),
            "committed_street": state.committed_street,
            "call_amount": (state.current_bet - actor_committed).clamp_min(0.0), "current_bet": state.current_bet,
            "min_raise_to": lower, "max_raise_to": upper, "last_full_raise": state.last_full_raise,
            "legal_action_mask": legality.mask, "raise_ticks": raise_ticks,
            "history": {name: getattr(history, name) for name in history.__dataclass_fields__},
        }
        compatible = ~(self.combo_cards[None, :, :, None].eq(board[:, None, None, :])
                       & board[:, None, None, :].ge(0)).any(3).any(2)
        return public, compatible

    @staticmethod
    def _ranges(log_reach: Tensor) -> Tensor:
        """model.py:285-287: each seat's reach over its private rows, normalised to a maximum of 1."""

        finite = torch.isfinite(log_reach)
        gauge = log_reach.masked_fill(~finite, -torch.inf).max(2, keepdim=True).values
        return torch.exp(log_reach - gauge).masked_fill(~finite, 0.0)

    @staticmethod
    def _evaluation(result: PolicyOutput) -> ModelEvaluation:
        """model.py:180-189."""

        if (result.t is None) != (result.c is None):
            raise PokerModelError("partition returned only one public branch head")
        public = MappingProxyType({}) if result.t is None else MappingProxyType({"trace": result.t, "cost": result.c})
        return ModelEvaluation(MappingProxyType(dict(result.raw)), result.v, public)

    # ------------------------------------------------------------ partitions
    def _call_preflop(self, model_input: Tensor, selected_private: Tensor | None = None) -> ModelEvaluation:
        """model.py:275-295."""

        state = self._state("pre", model_input)
        log_reach, history = self.machine.model_context("pre", model_input)
        public, _ = self._public(state, history)
        return self._evaluation(self.pre.forward_output(public, self._ranges(log_reach), None, public["to_act"],
                                                        selected_private=selected_private))

    def _call_postflop(self, input_type: str, model_input: Tensor,
                       selected_private: Tensor | None = None) -> ModelEvaluation:
        """model.py:297-350."""

        g = self.geometry
        state = self._state(input_type, model_input)
        log_reach, history = self.machine.model_context(input_type, model_input)
        public, compatible = self._public(state, history)
        live = int(input_type[5:])
        seats = torch.arange(g.players, device=state.device)[None].expand(state.rows, -1)
        ordered = torch.where(state.status.ne(FOLDED), seats, g.players).sort(1).values
        live_ids = ordered[:, :live]
        _assert(live_ids.lt(g.players).all(), "postflop family disagrees with live-seat state")
        ranges = self._ranges(log_reach)
        summary = unpack_folded_statistics(
            g, model_input[:, g.postflop_base_model_input_width:].float(), beta_rank=self.cfg.folder_beta_rank,
            line_metadata=fold_line_metadata(history, state.status, line_dim=self.cfg.folder_line_dim,
                                             stack_bb=g.stack_bb),
            status=state.status)
        masks = PostflopMasks(compatibility=compatible, seat_mask=public["seat_mask"], combo_mask=ranges.bool(),
                              status=public["status"], evaluator_summary=summary, live_seat_ids=live_ids)
        return self._evaluation(self.post.forward_output(public, ranges, public["to_act"], masks,
                                                         selected_private=selected_private))

    def _validate_output(self, evaluation: ModelEvaluation, batch: int, width: int, device) -> None:
        """model.py:109-144."""

        if evaluation.value.shape != (batch, width) or evaluation.value.device != device:
            raise PokerModelError("partition value output has the wrong domain")
        raw = evaluation.policy_raw
        if set(raw) != {"type_logits", "omega", "mu", "s", "iota"}:
            raise PokerModelError("partition policy output has unknown or missing fields")
        if raw["type_logits"].shape != (batch, width, 3):
            raise PokerModelError("partition type logits have the wrong domain")
        shape = raw["omega"].shape
        if (len(shape) != 3 or shape[:2] != (batch, width) or raw["mu"].shape != shape or raw["s"].shape != shape
                or raw["iota"].shape != (batch, width)):
            raise PokerModelError("partition raise outputs have the wrong domain")
        heads = evaluation.public_heads
        if heads and (set(heads) != {"trace", "cost"} or any(v.shape != (batch,) for v in heads.values())):
            raise PokerModelError("partition trace/cost outputs have the wrong shape")

    def forward_partition(self, input_type: str, model_input: Tensor,
                          selected_private: Tensor | None = None) -> ModelEvaluation:
        """model.py:352-387: K-wide preflop or H-wide postflop outputs (one row with ``selected_private``)."""

        if not model_input.is_cuda or model_input.ndim != 2 or not model_input.is_floating_point():
            raise PokerModelError("queued poker model input must be accelerator [B,F]")
        batch = model_input.shape[0]
        g = self.geometry
        if input_type == "pre":
            result = self._call_preflop(model_input, selected_private)
            width = g.private_classes
        elif input_type.startswith("post_") and input_type[5:].isdigit():
            if not 2 <= int(input_type[5:]) <= g.players:
                raise PokerModelError("postflop family has an invalid live-seat count")
            result = self._call_postflop(input_type, model_input, selected_private)
            width = g.private_hands
        else:
            raise PokerModelError(f"unknown poker input partition {input_type!r}")
        self._validate_output(result, batch, width if selected_private is None else 1, model_input.device)
        return result

    def forward_natural_partition(self, input_type: str, model_input: Tensor) -> ModelEvaluation:
        return self.forward_partition(input_type, model_input)

    def forward_sequential_partition(self, input_type: str, model_input: Tensor) -> ModelEvaluation:
        return self.forward_partition(input_type, model_input)

    def learner_operation(self, input_type: str, model_input: Tensor, sampled_private_state: Tensor,
                          owner: Tensor) -> ModelEvaluation:
        """model.py:403-415: the owner's sampled private row (its class preflop)."""

        combo = sampled_private_state.gather(1, owner.to(torch.int64)[:, None]).squeeze(1).to(torch.int64)
        index = self.combo_class.index_select(0, combo) if input_type == "pre" else combo
        return self.forward_partition(input_type, model_input, index)

    def rollout_operation(self, input_type: str, model_input: Tensor, _private_state: Tensor,
                          _owner: Tensor) -> ModelEvaluation:
        return self.forward_sequential_partition(input_type, model_input)

    def rb_learner_operation(self, input_type: str, model_input: Tensor, _private_state: Tensor,
                             _owner: Tensor) -> ModelEvaluation:
        return self.forward_natural_partition(input_type, model_input)

    def forward(self, input_type: str, model_input: Tensor, _private_state: Tensor, _owner: Tensor, *,
                natural_domain: bool = False) -> ModelEvaluation:
        """model.py:435-452."""

        if type(natural_domain) is not bool:
            raise TypeError("natural_domain must be bool")
        return (self.forward_natural_partition(input_type, model_input) if natural_domain
                else self.forward_sequential_partition(input_type, model_input))

    __call__ = forward


def parameter_shapes(cfg: PreflopConfig, rank_count: int, branching_heads: bool = False) -> dict[str, tuple[int, ...]]:
    """The reference QueuedPokerModel's parameter names and shapes (``shared.*``, ``pre_encoder.*``,
    ``post_encoder.*``; model.py:150-164), with the public branching heads when the mode is branched."""

    from .postflop import parameter_shapes as post_shapes
    from .preflop import parameter_shapes as pre_shapes

    pre = pre_shapes(cfg, rank_count)
    shared = {k: v for k, v in pre.items() if not k.startswith(("class_embedding", "class_row_affine"))}
    shapes = {f"shared.{k}": v for k, v in shared.items()}
    heads = {}
    if branching_heads:
        d, h = cfg.d_model, cfg.hidden
        public = (2 + cfg.max_players) * d
        for name, fan_in in (("public_features", public), ("t_features", d), ("c_features", d)):
            heads.update({f"branching_heads.{name}.w1.weight": (h, fan_in), f"branching_heads.{name}.w1.bias": (h,),
                          f"branching_heads.{name}.w2.weight": (d, h), f"branching_heads.{name}.w2.bias": (d,)})
        for name in ("t_affine", "c_affine"):
            heads.update({f"branching_heads.{name}.weight": (1, d), f"branching_heads.{name}.bias": (1,)})
    for family, table in (("pre_encoder", pre), ("post_encoder", post_shapes(cfg, rank_count))):
        shapes.update({f"{family}.{k}": v for k, v in table.items() if k not in shared})
        shapes.update({f"{family}.{k}": v for k, v in heads.items()})
    return shapes


__all__ = ["ModelEvaluation", "PokerModelError", "QueuedPokerModel", "fold_line_metadata", "parameter_shapes"]
