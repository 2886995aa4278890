"""The compact postflop combo-row policy/value network on this build's kernels.

``PostflopModel.forward`` computes pbg/games/poker/model/postflop.py:538-784
(``PostflopEncoder.forward``) with the shared trunk and readout of
pbg/games/poker/model/shared.py, from the reference's own parameters (the
``state_dict`` names of SharedPokerParameters and PostflopEncoder).  The trunk
(incidence residual, LayerNorm, biased attention, FamilyFFN with the "post"
static adapter) and the readout are the ones ``FamilyModel`` binds to
``pbg_linear_bf16`` / ``pbg_layernorm`` / ``pbg_attention_bf16``; this module
adds the postflop token assembly: the compact map over board-compatible combo
rows (incidence.py:87-216), combo embeddings, the evaluator-derived folded
geometry and folder context (postflop.py:104-346), the public tokens with board
cards and fold-line scalars (postflop.py:455-536), and the folded-seat summary
and compact scatter of the outputs.  Every FFN and affine map of width above 8
runs on the tensor-core GEMM; the 1-wide affine maps and the reductions are torch
operations on the device.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import torch
from torch import Tensor
from torch.nn import functional as F

from .checks import _assert, input_errors, raise_input_errors
from .preflop import FamilyModel, PolicyOutput, PreflopConfig, _affine_rows, lookup


@dataclass
class PostflopMasks:
    """postflop.py:34-52: the representation-boundary inputs of the compact encoder."""

    compatibility: Tensor
    seat_mask: Tensor | None = None
    combo_mask: Tensor | None = None
    status: Tensor | None = None
    combo_embeddings: Tensor | None = None
    evaluator_summary: object | None = None
    fold_line_features: Tensor | None = None
    live_seat_ids: Tensor | None = None
    compact_size: int | None = None


@dataclass
class CompactMap:
    """incidence.py:87-108: ``compact_to_full``/``valid`` [B,Q], ``full_to_compact`` [B,H] (-1 = omitted)."""

    compact_to_full: Tensor
    full_to_compact: Tensor
    valid: Tensor

    @property
    def batch_size(self) -> int:
        return self.compact_to_full.shape[0]

    @property
    def compact_size(self) -> int:
        return self.compact_to_full.shape[1]

    @property
    def full_size(self) -> int:
        return self.full_to_compact.shape[1]


def build_compact_map(compatibility: Tensor, compact_size: int | None = None) -> CompactMap:
    """incidence.py:111-149: a stable padded map of the supplied rows, in row order (no host read)."""

    if not isinstance(compatibility, Tensor) or compatibility.ndim != 2:
        raise ValueError("compatibility must have shape [B,H]")
    if compatibility.dtype != torch.bool:
        raise TypeError("compatibility must have dtype torch.bool")
    batch, full = compatibility.shape
    counts = compatibility.sum(1)
    q = full if compact_size is None else compact_size
    if isinstance(q, bool) or not 0 <= q <= full:
        raise ValueError("compact_size must be in [0,H]")
    _assert((counts <= q).all(), "compact_size omits compatible rows")
    rank = compatibility.long().cumsum(1) - 1
    full_to_compact = torch.where(compatibility, rank, torch.full_like(rank, -1))
    compact_to_full = torch.zeros((batch, q), dtype=torch.long, device=compatibility.device)
    if q:
        ids = torch.arange(full, device=compatibility.device)[None].expand(batch, -1)
        compact_to_full.scatter_add_(1, rank.clamp(0, q - 1), torch.where(compatibility, ids, torch.zeros_like(ids)))
    valid = torch.arange(q, device=compatibility.device)[None] < counts[:, None]
    return CompactMap(compact_to_full, full_to_compact, valid)


def _moved(values: Tensor, dim: int):
    dim = dim % values.ndim
    if dim == 0:
        raise ValueError("the batch dimension cannot be gathered or scattered")
    order = [0, dim] + [a for a in range(1, values.ndim) if a != dim]
    return values.permute(order), [order.index(a) for a in range(values.ndim)], dim


def compact_gather(values: Tensor, mapping: CompactMap, dim: int = 1) -> Tensor:
    """incidence.py:152-177: full rows -> padded compact rows (padding reads as zero)."""

    if not isinstance(values, Tensor) or values.ndim < 2:
        raise ValueError("values must have a batch and full-row dimension")
    moved, inverse, dim = _moved(values, dim)
    if values.shape[0] != mapping.batch_size or values.shape[dim] != mapping.full_size:
        raise ValueError("values do not match the compact map")
    tail = (1,) * (moved.ndim - 2)
    index = mapping.compact_to_full.reshape(mapping.batch_size, mapping.compact_size, *tail)
    out = moved.gather(1, index.expand(mapping.batch_size, mapping.compact_size, *moved.shape[2:]))
    return out.masked_fill(~mapping.valid.reshape(mapping.batch_size, mapping.compact_size, *tail), 0).permute(inverse)


def compact_scatter(values: Tensor, mapping: CompactMap, dim: int = 1, *, fill_value: float | bool = 0) -> Tensor:
    """incidence.py:180-216: padded compact rows -> the full row width (omitted rows = ``fill_value``)."""

    if not isinstance(values, Tensor) or values.ndim < 2:
        raise ValueError("values must have a batch and compact-row dimension")
    moved, inverse, dim = _moved(values, dim)
    if values.shape[0] != mapping.batch_size or values.shape[dim] != mapping.compact_size:
        raise ValueError("values do not match the compact map")
    suffix = moved.shape[2:]
    tail = (1,) * len(suffix)
    if not mapping.compact_size:
        return torch.full((mapping.batch_size, mapping.full_size, *suffix), fill_value, dtype=values.dtype,
                          device=values.device).permute(inverse)
    index = mapping.full_to_compact.clamp_min(0).reshape(mapping.batch_size, mapping.full_size, *tail)
    out = moved.gather(1, index.expand(mapping.batch_size, mapping.full_size, *suffix))
    selected = (mapping.full_to_compact >= 0).reshape(mapping.batch_size, mapping.full_size, *tail)
    return out.masked_fill(~selected, fill_value).permute(inverse)


def _fields(summary: object | None) -> Mapping | None:
    if hasattr(summary, "fields"):
        fields = summary.fields
        if not isinstance(fields, Mapping):
            raise TypeError("evaluator summary fields must be a mapping")
        return fields
    return summary if isinstance(summary, Mapping) else None


class PostflopModel(FamilyModel):
    """The postflop family (postflop.py:58-784): live seats x compact combo rows, FamilyFFN "post"."""

    family = "post"

    def __init__(self, cfg: PreflopConfig, rank_count: int, params: dict[str, Tensor], device) -> None:
        if cfg.folder_beta_rank > 4 * rank_count:
            raise ValueError("folder_beta_rank cannot exceed the active compact deck size")
        super().__init__(cfg, rank_count, params, device)
        lin, p = self._lin, self.p

        def ffn(name):
            return (lin(name + ".w1"), lin(name + ".w2"), name)

        self.combo_features = ffn("combo_features")
        self.folder_context = ffn("folder_context")
        self.fold_features = ffn("fold_features")
        self.row_affine = lin("row_affine")
        self.board_projection = lin("board_projection")
        self.tight_delta_projection = lin("tight_delta_projection", False)
        self.first_card = 52 - self.n_cards
        deck = torch.arange(self.first_card, 52)
        pairs = torch.combinations(deck, 2)  # lexicographic (a < b), the DeckGeometry combo order
        self.n_hands = pairs.shape[0]
        self.combo_cards = pairs.to(self.device)
        self.combo_ordinals = (pairs - self.first_card).to(self.device)
        two_hot = torch.zeros((self.n_hands, self.n_cards), dtype=torch.float32)
        two_hot.scatter_(1, pairs - self.first_card, 1.0)
        self.combo_two_hot = two_hot.to(self.device)

    # ------------------------------------------------------------ token assembly
    def _card_embedding(self, cards: Tensor) -> Tensor:
        """postflop.py:348-350: rank + suit embedding of global card ids (padding clamps to card 0)."""

        safe = cards.clamp(0, 51).long()
        return lookup(self.p["rank_embedding.weight"], safe // 4) + lookup(self.p["suit_embedding.weight"], safe % 4)

    def _combo_embedding(self, ids: Tensor, supplied: Tensor | None) -> Tensor:
        """postflop.py:352-365."""

        batch = ids.shape[0]
        if supplied is not None:
            expected = (self.n_hands, self.cfg.class_embedding_dim)
            if supplied.shape == expected:
                supplied = supplied[None].expand(batch, -1, -1)
            if supplied.shape != (batch,) + expected:
                raise ValueError("combo_embeddings has the wrong compact hand width")
            supplied = supplied.to(device=ids.device, dtype=torch.float32)
            return supplied.gather(1, ids[..., None].expand(-1, -1, supplied.shape[-1]))
        cards = self.combo_cards[ids]
        first, second = self._card_embedding(cards[..., 0]), self._card_embedding(cards[..., 1])
        return self._ffn(self.combo_features, torch.cat((first, second, first * second), -1)).float()

    def _folded_geometry(self, summary, mapping: CompactMap) -> tuple[Tensor, Tensor]:
        """postflop.py:104-175: hand log ratios and [two-hot | signed beta coordinates] per compact row."""

        batch, q = mapping.batch_size, mapping.compact_size
        dev = mapping.compact_to_full.device
        ids = mapping.compact_to_full
        cards = self.combo_ordinals[ids]
        geometry = self.combo_two_hot[ids]
        fields = _fields(summary)
        hand = None if fields is None else fields.get("hand_log_ratio")
        if hand is not None:
            if hand.shape != (batch, mapping.full_size):
                raise ValueError("hand_log_ratio must have shape [B,H]")
            lam = compact_gather(hand.to(device=dev, dtype=torch.float32), mapping, dim=1)
        elif fields is None:
            lam = torch.zeros((batch, q), device=dev)
        else:
            raise ValueError("current evaluator summaries require hand_log_ratio")
        rank = self.cfg.folder_beta_rank
        if rank:
            signed = torch.zeros((batch, q, 2 * rank), device=dev)
            if fields is not None:
                value, vector = fields.get("beta_eigenvalue"), fields.get("beta_eigenvector")
                if value is None or vector is None:
                    raise ValueError("current evaluator summaries require beta eigenvalue/vector fields")
                if value.shape[0] != batch or value.shape[1] < rank:
                    raise ValueError("beta_eigenvalue has insufficient rank")
                if vector.shape != (batch, self.n_cards, value.shape[1]):
                    raise ValueError("beta_eigenvector has the wrong shape")
                value = value[:, :rank].to(device=dev, dtype=torch.float32)
                vector = vector[:, :, :rank].to(device=dev, dtype=torch.float32)
                first = vector.gather(1, cards[..., 0, None].expand(-1, -1, rank))
                second = vector.gather(1, cards[..., 1, None].expand(-1, -1, rank))
                coordinate = (first + second) * value.abs().sqrt()[:, None, :]
                negative_axis = (value < 0)[:, None, :]
                signed = torch.cat((coordinate.masked_fill(negative_axis, 0.0),
                                    coordinate.masked_fill(~negative_axis, 0.0)), -1)
            geometry = torch.cat((geometry, signed), -1)
        lam = lam.masked_fill(~mapping.valid, 0.0)
        geometry = geometry.masked_fill(~mapping.valid[..., None], 0.0)
        return lam, geometry

    def _folder_context(self, summary, mapping: CompactMap, players: int, board: Tensor):
        """postflop.py:177-346: per-row card pressure, per-seat folder context and tight pair products."""

        d, eps = self.cfg.d_model, self.cfg.eps
        fields = _fields(summary)
        batch, q = mapping.batch_size, mapping.compact_size
        dev = mapping.compact_to_full.device
        empty_rows = torch.zeros((batch, q, d), device=dev)
        seat_context = torch.zeros((batch, players, d), device=dev)
        if fields is None or "folder_log_mass" not in fields:
            return empty_rows, seat_context, empty_rows
        log_mass = fields["folder_log_mass"].to(device=dev, dtype=torch.float32)
        folders = log_mass.shape[1]
        single, line = fields.get("folder_single_card_log_ratio"), fields.get("folder_line_meta")
        mask, seat = fields.get("folder_mask"), fields.get("folder_seat")
        valid, card_mass = fields.get("folder_output_valid"), fields.get("folder_card_mass")
        supplied_delta = fields.get("folder_delta")
        if card_mass is None and (single is None or single.shape != (batch, folders, self.n_cards)):
            raise ValueError("folder card marginals or single-card ratios are required")
        if card_mass is not None and card_mass.shape != (batch, folders, self.n_cards):
            raise ValueError("folder_card_mass has the wrong deck width")
        if line is None or line.shape != (batch, folders, self.cfg.folder_line_dim):
            raise ValueError("folder_line_meta has the wrong shape")
        if mask is None or mask.shape != (batch, folders) or mask.dtype != torch.bool:
            raise TypeError("folder_mask must be bool [B,F]")
        if valid is not None:
            if valid.shape != mask.shape or valid.dtype != torch.bool:
                raise TypeError("folder_output_valid must be bool [B,F]")
            mask = mask & valid
        mask = mask.to(dev)
        if single is not None:
            marginal = (1.0 - single.to(device=dev, dtype=torch.float32).exp()).clamp(0.0, 1.0)
        else:
            marginal = card_mass.to(device=dev, dtype=torch.float32) / log_mass.exp().clamp_min(eps)[..., None]
        context = self._ffn(self.folder_context,
                            torch.cat((log_mass[..., None], line.to(device=dev, dtype=torch.float32)), -1)).float()
        context = context * mask[..., None]
        if card_mass is None:
            unnormalized = log_mass.exp()[..., None] * marginal * mask[..., None]
        else:
            unnormalized = card_mass.to(device=dev, dtype=torch.float32) * mask[..., None]
        card_pressure = torch.einsum("bfc,bfd->bcd", unnormalized, context)
        cards = self.combo_ordinals[mapping.compact_to_full]
        pressure = (card_pressure.gather(1, cards[..., 0, None].expand(-1, -1, d))
                    + card_pressure.gather(1, cards[..., 1, None].expand(-1, -1, d)))
        folder_pool = context * unnormalized.sum(2, keepdim=True)
        if seat is not None:
            if seat.shape != (batch, folders):
                raise ValueError("folder_seat must have shape [B,F]")
            safe_seat = seat.to(device=dev, dtype=torch.long).clamp(0, players - 1)
            seat_context = seat_context.scatter_add(1, safe_seat[..., None].expand(-1, -1, d), context + folder_pool)
        board_ordinal = (board - self.first_card).clamp(0, self.n_cards - 1).long()
        on_board = (board_ordinal[..., None] == torch.arange(self.n_cards, device=dev)) & (board >= 0)[..., None]
        available = ~on_board.any(1)
        real = (board >= 0).sum(1)
        uniform = available.float() * (2.0 / (self.n_cards - real).float())[:, None]
        if supplied_delta is not None:
            if supplied_delta.shape != (batch, folders, self.n_cards):
                raise ValueError("folder_delta has the wrong deck width")
            delta = supplied_delta.to(device=dev, dtype=torch.float32) * mask[..., None]
        else:
            delta = (marginal - uniform[:, None, :]) * mask[..., None]
        projected = self.tight_delta_projection(delta).float()
        pair_products = 0.5 * (projected.sum(1).square() - projected.square().sum(1))
        tight_scalar = fields.get("tight_cluster_scalar")
        if tight_scalar is not None:
            if tight_scalar.shape != (batch,):
                raise ValueError("tight_cluster_scalar must have shape [B]")
            w = self.p["tight_contraction_projection.weight"][:, 0]
            pair_products = pair_products + tight_scalar.to(device=dev, dtype=torch.float32)[:, None] * w
        invalid = ~mapping.valid[..., None]
        pressure = pressure.masked_fill(invalid, 0.0)
        tight = pair_products[:, None, :].expand(-1, q, -1).masked_fill(invalid, 0.0)
        return pressure, seat_context, tight

    def _validate(self, pub: dict, ranges: Tensor, actor_seat: Tensor | None, masks: PostflopMasks):
        """postflop.py:367-453: actor, live seats, combo masks and the compact map."""

        if ranges.ndim != 3 or ranges.shape[-1] != self.n_hands or not ranges.is_floating_point():
            raise ValueError(f"combo_ranges must be floating point [B,P,{self.n_hands}]")
        batch, players = ranges.shape[:2]
        dev = ranges.device
        if players > self.cfg.max_players:
            raise ValueError("combo_ranges has more seats than max_players")
        compat = masks.compatibility
        if compat.shape != (batch, self.n_hands) or compat.dtype != torch.bool:
            raise TypeError(f"compatibility must be bool [B,{self.n_hands}]")
        if compat.device != dev:
            raise ValueError("compatibility and ranges must share a device")
        actor = (pub["to_act"] if actor_seat is None else actor_seat).to(device=dev, dtype=torch.long)
        if actor.shape != (batch,):
            raise ValueError("actor_seat must contain a valid seat for each batch row")
        _assert(((actor >= 0) & (actor < players)).all(), "actor_seat must contain a valid seat for each batch row")
        seat_mask = masks.seat_mask if masks.seat_mask is not None else pub.get("seat_mask")
        if seat_mask is None:
            seat_mask = torch.ones((batch, players), dtype=torch.bool, device=dev)
        if seat_mask.shape != (batch, players) or seat_mask.dtype != torch.bool:
            raise TypeError("seat_mask must be bool [B,P]")
        status = masks.status if masks.status is not None else pub.get("status")
        if status is None:
            status = torch.zeros((batch, players), dtype=torch.long, device=dev)
        status = status.to(device=dev, dtype=torch.long)
        if status.shape != (batch, players):
            raise ValueError("status must contain ids in [0,2]")
        _assert(((status >= 0) & (status <= 2)).all(), "status must contain ids in [0,2]")
        seat_mask = seat_mask & (status != 1)
        _assert(seat_mask.gather(1, actor[:, None]).all(), "the actor seat must be present")
        combo_mask = masks.combo_mask
        if combo_mask is None:
            combo_mask = compat[:, None, :].expand(-1, players, -1)
        if combo_mask.shape != ranges.shape or combo_mask.dtype != torch.bool:
            raise TypeError("combo_mask must be bool with the range shape")
        combo_mask = combo_mask & compat[:, None, :] & seat_mask[:, :, None]
        _assert(combo_mask[torch.arange(batch, device=dev), actor].any(1).all(),
                "each actor must have at least one compatible combo row")
        live_ids = masks.live_seat_ids
        if live_ids is None:
            seats = torch.arange(players, device=dev)[None].expand(batch, -1)
            ordered = torch.where(seat_mask, seats, players).sort(1).values
            live_valid = ordered < players
            live_ids = ordered.clamp_max(players - 1)
        else:
            if live_ids.ndim != 2 or live_ids.shape[0] != batch:
                raise ValueError("live_seat_ids must have shape [B,L]")
            live_ids = live_ids.to(device=dev, dtype=torch.long)
            _assert(((live_ids >= 0) & (live_ids < players)).all(), "live_seat_ids contains an invalid table seat")
            live_valid = seat_mask.gather(1, live_ids)
        _assert(((live_ids == actor[:, None]) & live_valid).any(1).all(), "live_seat_ids must contain each actor")
        return actor, seat_mask, live_ids, live_valid, status, combo_mask, build_compact_map(compat, masks.compact_size)

    def _public_tokens(self, pub: dict, fold: Tensor | None, relative: Tensor):
        """postflop.py:455-536: [state | scalars (+ fold-line moments) | board cards | history]."""

        p, dev, d = self.p, self.device, self.cfg.d_model
        batch, players = pub["stacks"].shape
        groups = [pub["pot"][:, None], pub["stacks"], pub["committed"], pub["street"].float()[:, None],
                  pub["legality_summary"].float(), pub["n_ticks"].float()[:, None], pub["raise_grid_bounds"].float()]
        kinds = [(1, 0), (players, 1), (players, 2), (1, 3), (pub["legality_summary"].shape[1], 4), (1, 5), (2, 6)]
        if pub.get("committed_street") is not None:
            groups.append(pub["committed_street"].float())
            kinds.append((players, 7))
        exact = [pub[k].float()[:, None] for k in ("call_amount", "current_bet", "min_raise_to", "max_raise_to",
                                                  "last_full_raise") if pub.get(k) is not None]
        if exact:
            groups.append(torch.cat(exact, 1))
            kinds.append((len(exact), 8))
        if pub.get("legal_action_mask") is not None:
            groups.append(pub["legal_action_mask"].float())
            kinds.append((pub["legal_action_mask"].shape[1], 9))
        if pub.get("raise_ticks") is not None:
            groups.append(pub["raise_ticks"].float())
            kinds.append((pub["raise_ticks"].shape[1], 10))
        if fold is not None:
            if fold.shape[0] != batch or not fold.is_floating_point():
                raise ValueError("fold_line_features must be floating point with leading B")
            flat = fold.flatten(1).float()
            groups.extend((flat.mean(1, keepdim=True), flat.square().mean(1, keepdim=True)))
            kinds.append((2, 11))
        scalars = torch.cat([g.float() for g in groups], 1)
        type_ids = torch.cat([torch.full((n,), k, dtype=torch.long, device=dev) for n, k in kinds])
        token = (scalars[..., None] * p["public_scalar_affine.weight"][:, 0] + p["public_scalar_affine.bias"]
                 + lookup(p["public_type_embedding.weight"], type_ids))
        seat_pos = lookup(p["seat_embedding.weight"], relative)
        rest = scalars.shape[1] - 1 - 2 * players
        zeros = torch.zeros((batch, 1, d), device=dev)
        token = token + torch.cat((zeros, seat_pos, seat_pos, zeros.expand(-1, rest, -1)), 1)
        board = pub["board"]
        board_tokens = self.board_projection(self._card_embedding(board)).float() + p["public_type_embedding.weight"][12]
        state = p["state_token"].expand(batch, 1, d)
        supplied = pub.get("seat_mask")
        supplied = torch.ones((batch, players), dtype=torch.bool, device=dev) if supplied is None else supplied.bool()
        ones = lambda n: torch.ones((batch, n), dtype=torch.bool, device=dev)  # noqa: E731
        tokens = torch.cat((state, token, board_tokens), 1)
        valid = torch.cat((ones(2), supplied, supplied, ones(rest), board >= 0), 1)
        h = pub.get("history")
        if h is not None and h["mask"].shape[1]:
            if h["mask"].shape[1] > self.cfg.max_history_tokens:
                raise ValueError("public history exceeds max_history_tokens")
            numeric = torch.stack([h[k].float() for k in ("amount", "pot_before", "call_amount", "current_bet",
                                                          "min_raise_to", "max_raise_to")], -1)
            ht = numeric @ p["history_numeric_affine.weight"].T + p["history_numeric_affine.bias"]
            ht = ht + lookup(p["history_action_embedding.weight"], h["action"].clamp(0, 3).long())
            ht = ht + lookup(p["history_street_embedding.weight"], h["street"].clamp(0, 3).long())
            ht = ht + p["history_position_embedding.weight"][: h["mask"].shape[1]][None]
            actor = h["actor"].clamp(0, players - 1).long()
            ht = ht + lookup(p["seat_embedding.weight"], relative.gather(1, actor)) * (h["actor"] >= 0)[..., None]
            tokens = torch.cat((tokens, ht), 1)
            valid = torch.cat((valid, h["mask"].bool()), 1)
        return tokens, valid

    # ------------------------------------------------------------ forward
    def forward(self, pub: dict, combo_ranges: Tensor, actor_seat: Tensor | None = None,
                masks: PostflopMasks | None = None, *, selected_private: Tensor | None = None):
        """postflop.py:538-784 -> (raw policy fields over the full hand width [B,H,...], value [B,H]);
        with ``selected_private`` [B] the one selected row per decision ([B,1,...])."""

        out = self.forward_output(pub, combo_ranges, actor_seat, masks, selected_private=selected_private)
        return out.raw, out.v

    def forward_output(self, pub: dict, combo_ranges: Tensor, actor_seat: Tensor | None = None,
                       masks: PostflopMasks | None = None, *, selected_private: Tensor | None = None) -> PolicyOutput:
        """postflop.py:538-784 -> PolicyOutput(raw, v, t, c)."""

        if masks is None:
            raise ValueError("postflop forward requires supplied compatibility")
        cfg, p, d, eps = self.cfg, self.p, self.cfg.d_model, self.cfg.eps
        ranges = combo_ranges.to(self.device, torch.float32)
        actor, seat_mask, live_ids, live_valid, status, combo_mask, mapping = self._validate(
            pub, ranges, actor_seat, masks)
        dev = ranges.device
        batch, players = ranges.shape[:2]
        live = live_ids.shape[1]
        q = mapping.compact_size
        live_index = live_ids[..., None].expand(-1, -1, q)
        compact_ranges = compact_gather(ranges, mapping, dim=2).gather(1, live_index)
        compact_mask = compact_gather(combo_mask, mapping, dim=2).bool().gather(1, live_index) & live_valid[..., None]
        combo_emb = self._combo_embedding(mapping.compact_to_full, masks.combo_embeddings)
        lam, geometry = self._folded_geometry(masks.evaluator_summary, mapping)
        pressure, folder_seat_context, tight = self._folder_context(masks.evaluator_summary, mapping, players,
                                                                    pub["board"])
        log_range = torch.log(compact_ranges.clamp_min(eps))
        base = compact_ranges.masked_fill(~compact_mask, 0.0)
        base = base / base.sum(2, keepdim=True).clamp_min(eps)
        corrected = (torch.log(base.clamp_min(eps)) + lam[:, None, :]).masked_fill(~compact_mask, -torch.inf)
        normalizer = torch.logsumexp(corrected, 2, keepdim=True)
        corrected = torch.where(compact_mask, corrected - normalizer.masked_fill(~torch.isfinite(normalizer), 0.0),
                                torch.zeros_like(corrected))
        ex = lambda t: t[:, None].expand(-1, live, -1, -1)  # noqa: E731
        ones = torch.ones_like(compact_ranges)[..., None]
        feats = torch.cat((compact_ranges[..., None], log_range[..., None], corrected[..., None],
                           ex(combo_emb), ex(geometry), ex(pressure), ones), -1)
        seats = torch.arange(players, device=dev)[None].expand(batch, -1)
        button = pub.get("button")
        relative = torch.remainder(seats - button[:, None].long(), players) if button is not None else seats
        live_relative = relative.gather(1, live_ids)
        live_status = status.gather(1, live_ids)
        # each live seat's seat, status and actor embeddings, added to its q rows in the map's epilogue
        seat_terms = (lookup(p["seat_embedding.weight"], live_relative) + lookup(p["status_embedding.weight"], live_status)
                      + lookup(p["actor_embedding.weight"], (live_ids == actor[:, None]).long()))
        row = _affine_rows(self.row_affine, feats, seat_terms, q)
        rows_k = live * q
        public, public_mask = self._public_tokens(pub, masks.fold_line_features, relative)
        actor_relative = relative.gather(1, actor[:, None]).squeeze(1)
        anchors = p["anchor_tokens"][None] + lookup(p["anchor_seat_embedding.weight"], actor_relative)[:, None]
        x = torch.cat((row.reshape(batch, rows_k, d), public, anchors), 1)
        key_mask = torch.cat((compact_mask.reshape(batch, -1), public_mask,
                              torch.ones((batch, cfg.k_act), dtype=torch.bool, device=dev)), 1)
        key_bias = torch.cat((corrected.reshape(batch, -1),
                              torch.zeros((batch, x.shape[1] - rows_k), device=dev)), 1).contiguous()
        side = torch.cat((ex(combo_emb), compact_ranges[..., None], log_range[..., None], corrected[..., None],
                          ex(geometry), ex(geometry[..., self.n_cards:].square()), ex(pressure), ex(tight)), -1)
        incidence_mass = corrected.exp() * compact_mask
        identical_scale = torch.ones((batch, q), device=dev)

        x = self._trunk(x, live, q, incidence_mass, geometry[..., : self.n_cards].contiguous(), identical_scale,
                        side, key_bias, key_mask)
        final = self._ln(x, self.final_ln).float()
        final_rows = final[:, :rows_k].reshape(batch, live, q, d)
        final_public = final[:, rows_k: -cfg.k_act]
        final_anchors = final[:, -cfg.k_act:]
        public_valid = public_mask.float()
        public_mean = (final_public * public_valid[..., None]).sum(1) / public_valid.sum(1, keepdim=True)
        arange = torch.arange(batch, device=dev)
        actor_live = ((live_ids == actor[:, None]) & live_valid).long().argmax(1)
        actor_rows = final_rows[arange, actor_live]
        actor_mask = compact_mask[arange, actor_live]
        actor_anchor = torch.cat((final_anchors[:, 0], final_anchors[:, 1], final_anchors[:, 2],
                                  final_anchors[:, 3:].mean(1)), -1)
        actor_summary = self._ffn(self.actor_seat_features, actor_anchor).float()
        mass = incidence_mass.sum(2)
        pooled = (final_rows * incidence_mass[..., None]).sum(2) / mass[..., None].clamp_min(eps)
        scale = 1.0 / max(cfg.max_players - 1, 1)
        live_meta = torch.stack((mass, live_status.float() / 2.0, live_relative.float() * scale), -1)
        live_summary = self._ffn(self.seat_features, torch.cat((pooled, live_meta), -1)).float()
        full_mass = torch.zeros((batch, players), device=dev).scatter_add(1, live_ids, mass * live_valid.float())
        seat_meta = torch.stack((full_mass, status.float() / 2.0, relative.float() * scale), -1)
        folded_summary = self._ffn(self.fold_features, torch.cat((folder_seat_context, seat_meta), -1)).float()
        scattered = torch.zeros_like(folded_summary).scatter_add(1, live_ids[..., None].expand(-1, -1, d),
                                                                 live_summary * live_valid[..., None])
        seat_summary = torch.where(seat_mask[..., None], scattered, folded_summary)
        selector = torch.arange(players, device=dev)[None] == actor[:, None]
        seat_summary = torch.where(selector[..., None], actor_summary[:, None], seat_summary)
        supplied = pub.get("seat_mask")
        if supplied is not None:
            seat_summary = seat_summary.masked_fill(~supplied.bool()[..., None], 0.0)
        ordered = torch.zeros_like(seat_summary).scatter(1, relative[..., None].expand(-1, -1, d), seat_summary)
        padded = torch.cat((ordered, torch.zeros((batch, cfg.max_players - players, d), device=dev)), 1)
        global_feature = self._ffn(self.global_features,
                                   torch.cat((public_mean, actor_summary, padded.reshape(batch, -1)), -1)).float()
        if selected_private is not None:
            selected = mapping.full_to_compact.gather(1, selected_private.to(dev).long()[:, None])
            _assert(selected.ge(0).all(), "selected private hand is board-incompatible")
            actor_rows = actor_rows.gather(1, selected[..., None].expand(-1, 1, d))
            combo_emb = combo_emb.gather(1, selected[..., None].expand(-1, 1, cfg.class_embedding_dim))
            actor_mask = actor_mask.gather(1, selected)
        raw, value = self._readout(actor_rows, combo_emb, final_anchors, global_feature)
        raw = {k: v.masked_fill(~(actor_mask[..., None] if v.ndim == 3 else actor_mask), 0) for k, v in raw.items()}
        value = value.masked_fill(~actor_mask, 0)
        if selected_private is None:
            raw = {k: compact_scatter(v, mapping, dim=1) for k, v in raw.items()}
            full_mask = compact_scatter(actor_mask, mapping, dim=1)
            value = compact_scatter(value, mapping, dim=1)
        else:
            full_mask = actor_mask
        invalid = ~full_mask
        raw["omega"] = raw["omega"].masked_fill(invalid[..., None], 1.0 / cfg.m_raise)
        raw["mu"] = raw["mu"].masked_fill(invalid[..., None], 0.5)
        raw["s"] = raw["s"].masked_fill(invalid[..., None], 1.0)
        raw["iota"] = raw["iota"].masked_fill(invalid, 0.5)
        t, cost = self._branching(global_feature, public_mean, padded)
        return PolicyOutput(raw, value, t, cost)


def parameter_shapes(cfg: PreflopConfig, rank_count: int) -> dict[str, tuple[int, ...]]:
    """Names and shapes of the parameters PostflopModel binds: SharedPokerParameters (shared.py:36-72,
    as for the preflop family) and PostflopEncoder (postflop.py:64-96) without the branching heads."""

    from .preflop import parameter_shapes as shared_shapes

    d, dc, h = cfg.d_model, cfg.class_embedding_dim, cfg.hidden
    n_cards = 4 * rank_count
    shapes = {k: v for k, v in shared_shapes(cfg, rank_count).items()
              if not k.startswith(("class_embedding", "class_row_affine"))}
    geo = n_cards + 2 * cfg.folder_beta_rank
    shapes.update({"rank_embedding.weight": (13, dc), "suit_embedding.weight": (4, dc),
                   "row_affine.weight": (d, 3 + dc + geo + d + 1), "row_affine.bias": (d,),
                   "tight_delta_projection.weight": (d, n_cards), "tight_contraction_projection.weight": (d, 1),
                   "board_projection.weight": (d, dc), "board_projection.bias": (d,)})
    for name, (fan_in, out) in {"combo_features": (3 * dc, dc), "folder_context": (1 + cfg.folder_line_dim, d),
                                "fold_features": (d + 3, d)}.items():
        shapes.update({f"{name}.w1.weight": (h, fan_in), f"{name}.w1.bias": (h,),
                       f"{name}.w2.weight": (out, h), f"{name}.w2.bias": (out,)})
    return shapes


__all__ = ["CompactMap", "PostflopMasks", "PostflopModel", "build_compact_map", "compact_gather",
           "compact_scatter", "input_errors", "parameter_shapes", "raise_input_errors"]
