"""Multiway folded-range statistics (pbg/games/poker/queued/folded.py) on this build's kernel.

``folded_statistics`` returns the reference's summary mapping (Lambda_B per
private hand, the signed beta eigenpairs, folder log masses, card masses, line
metadata, masks, seats and the tight-cluster scalar) for the postflop model
input.  The finite-difference estimator over every zero-, one- and two-card
removal query (folded.py:111-232, the reference's dense chunked einsums) runs in
one launch of ``pbg_folded_phi_queries``; the eigendecomposition of the beta
matrices (the reference's ``torch.linalg.eigh``) runs in one launch of
``pbg_symmetric_eigh``; the range normalisation and the alpha / beta assembly
and card masses around them are torch operations on the device, as in the
reference.
"""

from __future__ import annotations

from collections.abc import Mapping
from types import MappingProxyType

import torch
from torch import Tensor

from ._native import NativeError, call, lib, ptr, stream
from .checks import _assert
from .poker import FOLDED, PAD_CARD, NLHEGeometry

_REMOVAL_QUERY_CHUNK = 64


class FoldedStatisticsError(ValueError):
    pass


def folded_statistics_workspace_row_bytes(geometry: NLHEGeometry) -> int:
    """folded.py:21-46: the per-row workspace bound the reference's admission control charges."""

    if geometry.players == 2:
        return 0
    cards, players, hands = geometry.deck_cards, geometry.players, geometry.private_hands
    queries = 1 + cards + cards * (cards - 1) // 2
    chunk = min(queries, _REMOVAL_QUERY_CHUNK)
    values = (players * cards * cards + chunk * (2 * players * cards + players * players + 8 * players + 8)
              + 2 * queries + 10 * chunk * hands + hands + 3 * cards * cards)
    return 4 * values


def sequential_family_workspace_row_bytes(geometry: NLHEGeometry, m_raise: int) -> int:
    """folded.py:49-76: model outputs, transition state and folded scratch of one family row."""

    if isinstance(m_raise, bool) or not isinstance(m_raise, int) or m_raise <= 0:
        raise ValueError("raise-mixture count must be positive")
    hands, players = geometry.private_hands, geometry.players
    width = geometry.postflop_model_input_width
    model = width + hands * (5 + 3 * m_raise)
    transition = 2 * width + 8 * players * hands + 4 * hands + 128 * players + 256
    return 4 * (model + transition) + folded_statistics_workspace_row_bytes(geometry)


def phi_queries(probability: Tensor, folder_mask: Tensor, tight_mask: Tensor, base_cards: Tensor,
                cards: int) -> tuple[Tensor, Tensor]:
    """folded.py:111-232 over every removal query: (phi + triple, triple), each f32 [B, 1 + C + C(C-1)/2]."""

    batch, players, hands = probability.shape
    if hands != cards * (cards - 1) // 2 or probability.dtype != torch.float32 or not probability.is_cuda:
        raise NativeError("folded phi queries take float32 CUDA probabilities [B,P,C(C-1)/2]")
    queries = int(lib().pbg_folded_query_count(cards))
    probability = probability.contiguous()
    folder = folder_mask.to(torch.uint8).contiguous()
    tight = tight_mask.to(torch.uint8).contiguous()
    base = base_cards.to(torch.float32).contiguous()
    phi = torch.empty((batch, queries), dtype=torch.float32, device=probability.device)
    triple = torch.empty_like(phi)
    call("pbg_folded_phi_queries", batch, players, cards, ptr(probability), ptr(folder), ptr(tight), ptr(base),
         ptr(phi), ptr(triple), stream(probability.device))
    return phi, triple


def symmetric_eigh(matrices: Tensor, max_sweeps: int = 20) -> tuple[Tensor, Tensor]:
    """torch.linalg.eigh's contract for a batch of small symmetric fp32 matrices [B, n, n] (n <= 64):
    eigenvalues ascending [B, n] and eigenvectors as columns [B, n, n], on pbg_symmetric_eigh (Jacobi,
    one CTA per matrix) instead of a library solver that takes the batch one matrix at a time."""

    if matrices.ndim != 3 or matrices.shape[1] != matrices.shape[2] or not matrices.is_cuda:
        raise NativeError("symmetric_eigh takes CUDA matrices [B, n, n]")
    batch, n, _ = matrices.shape
    source = matrices.to(torch.float32).contiguous()
    values = torch.empty((batch, n), dtype=torch.float32, device=source.device)
    vectors = torch.empty((batch, n, n), dtype=torch.float32, device=source.device)
    call("pbg_symmetric_eigh", batch, n, ptr(source), ptr(values), ptr(vectors), max_sweeps, stream(source.device))
    order = values.argsort(-1)
    return values.gather(1, order), vectors.gather(2, order[:, None].expand(-1, n, -1))


def _board_card_mask(board_cards: Tensor, board_valid: Tensor, first_card: int, cards: int) -> Tensor:
    """folded.py:330-336: each board slot's validity written at its clamped deck-local index in slot
    order (an empty slot, clamped to the last card, written after that card clears its mark)."""

    local = (board_cards.long() - first_card).clamp(0, cards - 1)
    hit = local[..., None] == torch.arange(cards, device=board_cards.device)          # [B,5,C]
    slot = torch.arange(1, board_cards.shape[1] + 1, device=board_cards.device)[None, :, None]
    last = (hit * slot).amax(1)                                                        # [B,C], 0 = never written
    written = board_valid.gather(1, (last - 1).clamp_min(0))
    return (last > 0) & written


def _folded_statistics_fp32(geometry: NLHEGeometry, *, board_cards: Tensor, range_weights: Tensor, status: Tensor,
                            combo_cards: Tensor, beta_rank: int, line_dim: int, line_metadata: Tensor | None = None,
                            tight_mask: Tensor | None = None) -> Mapping[str, Tensor]:
    """folded.py:235-392."""

    batch, players, hands = range_weights.shape
    cards = geometry.deck_cards
    if (board_cards.device.type != "cuda" or board_cards.shape != (batch, 5) or range_weights.dtype != torch.float32
            or status.shape != (batch, players) or hands != geometry.private_hands
            or combo_cards.shape != (hands, 2) or not 0 <= beta_rank <= cards or line_dim < 0
            or (line_dim > 0 and line_metadata is None)
            or (line_metadata is not None and (line_metadata.shape != (batch, players, line_dim)
                                               or line_metadata.dtype != torch.float32
                                               or line_metadata.device != range_weights.device))):
        raise FoldedStatisticsError("folded statistic inputs violate poker geometry")
    device = range_weights.device
    folder_mask = status.eq(FOLDED)
    if tight_mask is None:
        tight_mask = folder_mask
    if tight_mask.shape != folder_mask.shape or tight_mask.dtype != torch.bool or tight_mask.device != device:
        raise FoldedStatisticsError("tight-folder mask violates folded seats")
    _assert((~tight_mask | folder_mask).all(), "tight-folder mask includes a live seat")
    tiny = torch.finfo(torch.float32).tiny
    raw = range_weights.masked_fill(~torch.isfinite(range_weights), 0.0).clamp_min(0.0)
    raw = raw * folder_mask[..., None]
    board_valid = board_cards.ne(PAD_CARD)
    conflict = (board_valid[..., None, None] & board_cards.long()[..., None, None].eq(combo_cards[None])).any(1).any(-1)
    raw = raw.masked_fill(conflict[:, None], 0.0)
    mass = raw.sum(-1)
    probability = raw / mass.clamp_min(tiny)[..., None]
    base_cards = cards - board_valid.sum(-1, dtype=torch.float32)
    phi, triple = phi_queries(probability, folder_mask, tight_mask, base_cards, cards)

    combo_local = (combo_cards - geometry.first_card).to(torch.int64)
    pair = torch.triu_indices(cards, cards, offset=1, device=device)
    pair_ordinal = torch.arange(pair.shape[1], device=device) + 1 + cards
    phi_zero = phi[:, :1]
    alpha = phi[:, 1: 1 + cards] - phi_zero
    beta = torch.zeros((batch, cards, cards), dtype=torch.float32, device=device)
    pair_value = phi.index_select(1, pair_ordinal) - phi[:, 1 + pair[0]] - phi[:, 1 + pair[1]] + phi_zero
    beta[:, pair[0], pair[1]] = pair_value
    beta[:, pair[1], pair[0]] = pair_value
    on_board = _board_card_mask(board_cards, board_valid, geometry.first_card, cards)
    beta = beta.masked_fill(on_board[:, :, None] | on_board[:, None, :], 0.0)
    alpha = alpha.masked_fill(on_board, 0.0)
    hand_log_ratio = (alpha[:, combo_local[:, 0]] + alpha[:, combo_local[:, 1]]
                      + beta[:, combo_local[:, 0], combo_local[:, 1]])
    if beta_rank:
        eigenvalue, eigenvector = symmetric_eigh(beta)
        order = torch.argsort(eigenvalue.abs(), dim=-1, descending=True, stable=True)[:, :beta_rank]
        eigenvalue = eigenvalue.gather(1, order)
        eigenvector = eigenvector.gather(2, order[:, None].expand(-1, cards, -1))
        pivot = eigenvector.abs().argmax(1)
        orientation = eigenvector.gather(1, pivot[:, None]).squeeze(1)
        eigenvector = eigenvector * torch.where(orientation < 0, -1.0, 1.0)[:, None]
    else:
        eigenvalue = raw.new_zeros((batch, 0))
        eigenvector = raw.new_zeros((batch, cards, 0))
    incidence = raw.new_zeros((hands, cards))
    incidence.scatter_(1, combo_local, 1.0)
    card_mass = torch.einsum("bph,hc->bpc", raw, incidence)
    line_meta = raw.new_zeros((batch, players, line_dim)) if line_metadata is None else line_metadata * folder_mask[..., None]
    return MappingProxyType({
        "hand_log_ratio": hand_log_ratio.contiguous(),
        "beta_eigenvalue": eigenvalue.contiguous(),
        "beta_eigenvector": eigenvector.contiguous(),
        "folder_log_mass": torch.where(folder_mask, torch.log(mass.clamp_min(tiny)), torch.zeros_like(mass)).contiguous(),
        "folder_card_mass": card_mass.contiguous(),
        "folder_line_meta": line_meta.contiguous(),
        "folder_mask": folder_mask.contiguous(),
        "folder_output_valid": folder_mask.logical_and(mass > 0).contiguous(),
        "folder_seat": torch.arange(players, dtype=torch.int64, device=device)[None].expand(batch, -1).contiguous(),
        "tight_cluster_scalar": triple[:, 0].contiguous(),
    })


def folded_statistics(geometry: NLHEGeometry, *, board_cards: Tensor, range_weights: Tensor, status: Tensor,
                      combo_cards: Tensor, beta_rank: int, line_dim: int, line_metadata: Tensor | None = None,
                      tight_mask: Tensor | None = None) -> Mapping[str, Tensor]:
    """folded.py:395-419: the statistics outside mixed precision."""

    with torch.autocast(device_type="cuda", enabled=False):
        return _folded_statistics_fp32(geometry, board_cards=board_cards, range_weights=range_weights, status=status,
                                       combo_cards=combo_cards, beta_rank=beta_rank, line_dim=line_dim,
                                       line_metadata=line_metadata, tight_mask=tight_mask)


def pack_folded_statistics(geometry: NLHEGeometry, summary: Mapping[str, Tensor]) -> Tensor:
    """folded.py:422-450: the model-consumed fields packed into the retained family row."""

    batch = summary["hand_log_ratio"].shape[0]
    value = torch.cat((summary["hand_log_ratio"], summary["beta_eigenvalue"], summary["beta_eigenvector"].flatten(1),
                       summary["folder_log_mass"], summary["folder_card_mass"].flatten(1),
                       summary["tight_cluster_scalar"][:, None],
                       torch.ones((batch, 1), dtype=summary["hand_log_ratio"].dtype,
                                  device=summary["hand_log_ratio"].device)), 1).contiguous()
    if value.shape != (batch, geometry.folded_summary_width):
        raise FoldedStatisticsError("packed folded summary has the wrong width")
    return value


def unpack_folded_statistics(geometry: NLHEGeometry, packed: Tensor, *, beta_rank: int, line_metadata: Tensor,
                             status: Tensor) -> Mapping[str, Tensor]:
    """folded.py:453-530: the model view of a retained row, without recomputation."""

    batch = packed.shape[0]
    cards, hands, players = geometry.deck_cards, geometry.private_hands, geometry.players
    folder_mask = status.eq(FOLDED)
    seats = torch.arange(players, dtype=torch.int64, device=packed.device)[None].expand(batch, -1)
    if geometry.folded_summary_width == 0:
        return MappingProxyType({
            "hand_log_ratio": packed.new_zeros((batch, hands)),
            "beta_eigenvalue": packed.new_zeros((batch, beta_rank)),
            "beta_eigenvector": packed.new_zeros((batch, cards, beta_rank)),
            "folder_log_mass": packed.new_zeros((batch, players)),
            "folder_card_mass": packed.new_zeros((batch, players, cards)),
            "folder_line_meta": line_metadata * folder_mask[..., None],
            "folder_mask": folder_mask, "folder_output_valid": folder_mask, "folder_seat": seats,
            "tight_cluster_scalar": packed.new_zeros((batch,)),
        })
    if packed.shape != (batch, geometry.folded_summary_width):
        raise FoldedStatisticsError("retained folded summary has the wrong width")
    widths = (hands, cards, cards * cards, players, players * cards, 1, 1)
    parts = torch.split(packed, widths, dim=1)
    summary_valid = parts[6][:, 0].gt(0.5)
    _assert((~folder_mask.any(-1) | summary_valid).all(), "postflop folded seats require a sealed folded summary")
    return MappingProxyType({
        "hand_log_ratio": parts[0],
        "beta_eigenvalue": parts[1][:, :beta_rank],
        "beta_eigenvector": parts[2].reshape(batch, cards, cards)[:, :, :beta_rank],
        "folder_log_mass": parts[3],
        "folder_card_mass": parts[4].reshape(batch, players, cards),
        "folder_line_meta": line_metadata * folder_mask[..., None],
        "folder_mask": folder_mask, "folder_output_valid": folder_mask, "folder_seat": seats,
        "tight_cluster_scalar": parts[5][:, 0],
    })


__all__ = ["FoldedStatisticsError", "folded_statistics", "folded_statistics_workspace_row_bytes",
           "pack_folded_statistics", "phi_queries", "sequential_family_workspace_row_bytes", "symmetric_eigh",
           "unpack_folded_statistics"]
