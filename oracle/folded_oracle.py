"""numpy restatement of the multiway folded-range statistics (test infrastructure only).

Only ``tests/`` import this module; it is the checker for ``pbg_folded_phi_queries``
and ``pbg_b200.folded``, never part of the shipped path.  It follows
pbg/games/poker/queued/folded.py:

* ``removal_queries``   folded.py:81-92   (zero-, one- and two-card removals, pairs in triu order)
* ``phi_queries``       folded.py:111-232 (the estimator on every removal query)
* ``folded_statistics`` folded.py:235-392 (Lambda_B, signed beta eigenpairs, folder masses)
* ``workspace_row_bytes`` / ``family_workspace_row_bytes`` folded.py:21-76 (admission bounds)

It computes in float64 (the reference computes in float32), vectorised over the queries; the
float32 tiny that the reference clamps with is kept, and clamps propagate NaN as torch's do.
"""

from __future__ import annotations

import numpy as np

TINY = float(np.finfo(np.float32).tiny)
PAD_CARD = 255
FOLDED = 1
QUERY_CHUNK = 64


def combos(cards: int) -> np.ndarray:
    """Deck-local card pairs of every private hand, lexicographic (hooks.py:1128-1143)."""

    return np.array([(a, b) for a in range(cards) for b in range(a + 1, cards)], dtype=np.int64)


def removal_queries(cards: int) -> np.ndarray:
    """folded.py:81-92: query 0 removes nothing, 1..C one card, then every pair in triu order."""

    pairs = combos(cards)
    removal = np.zeros((1 + cards + len(pairs), cards), dtype=bool)
    removal[1: 1 + cards] = np.eye(cards, dtype=bool)
    rows = np.arange(len(pairs)) + 1 + cards
    removal[rows, pairs[:, 0]] = True
    removal[rows, pairs[:, 1]] = True
    return removal


def _clamp(x, low):
    return np.where(np.isnan(x), x, np.maximum(x, low))


def phi_queries(probability: np.ndarray, folder_mask: np.ndarray, tight_mask: np.ndarray,
                base_cards: float, removal: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """folded.py:111-232 for one decision: probability [F,H], masks [F], removal [Q,C] -> (phi+triple, triple)."""

    folders, hands = probability.shape
    cards = removal.shape[1]
    pair = combos(cards)
    matrix = np.zeros((folders, cards, cards))
    matrix[:, pair[:, 0], pair[:, 1]] = probability
    matrix[:, pair[:, 1], pair[:, 0]] = probability
    remove = removal.astype(np.float64)
    allowed = ~removal
    available = base_cards - remove.sum(-1)                                   # [Q]
    marginal = matrix.sum(-1)                                                 # [F,C]
    linear = remove @ marginal.T                                              # [Q,F]
    quadratic = 0.5 * np.einsum("qc,fcd,qd->qf", remove, matrix, remove)
    surviving = _clamp(1.0 - linear + quadratic, TINY)
    removed_column = np.einsum("fcd,qd->qfc", matrix, remove)
    conditional = (marginal[None] - removed_column) * allowed[:, None, :] / surviving[..., None]
    flat = 2.0 / np.maximum(available, 1.0)
    delta = conditional - flat[:, None, None] * allowed[:, None, :]
    with np.errstate(divide="ignore", invalid="ignore"):
        phi = (np.log(surviving) * folder_mask[None].astype(np.float64)).sum(-1)
        count = int(folder_mask.sum())
        denominator = available * (available - 1.0) * 0.5
        for packed in range(1, folders):
            numerator_cards = available - 2.0 * packed
            numerator = numerator_cards * (numerator_cards - 1.0) * 0.5
            if count > packed:
                phi = phi + np.log(_clamp(numerator / denominator, TINY))
        survives = (allowed[:, pair[:, 0]] & allowed[:, pair[:, 1]]).astype(np.float64)   # [Q,H]
        uniform_pair = _clamp(1.0 - 4.0 / available + 1.0 / denominator, TINY)
        for f in range(folders):
            for g in range(f + 1, folders):
                if folder_mask[f] and folder_mask[g]:
                    dot = (conditional[:, f] * conditional[:, g]).sum(-1)
                    identical = 2.0 * (survives @ (probability[f] * probability[g]))
                    identical = identical / (surviving[:, f] * surviving[:, g])
                    disjoint = _clamp(1.0 - dot + 0.5 * identical, TINY)
                    phi = phi + np.log(disjoint / uniform_pair)
    triple = np.zeros(len(removal))
    for f in range(folders):
        for g in range(f + 1, folders):
            if not (tight_mask[f] and tight_mask[g]):
                continue
            left, right = delta[:, f], delta[:, g]
            for hub in range(folders):
                if hub in (f, g) or not folder_mask[hub]:
                    continue
                edge = left[:, pair[:, 0]] * right[:, pair[:, 1]] + left[:, pair[:, 1]] * right[:, pair[:, 0]]
                matrix_term = (edge * survives * probability[hub][None]).sum(-1) / surviving[:, hub]
                hub_marginal = conditional[:, hub]
                diagonal = (hub_marginal * left * right).sum(-1)
                outer = (hub_marginal * left).sum(-1) * (hub_marginal * right).sum(-1)
                triple = triple + matrix_term + diagonal - outer
    return phi + triple, triple


def folded_statistics(board_cards: np.ndarray, range_weights: np.ndarray, status: np.ndarray, ranks: int,
                      beta_rank: int, line_metadata: np.ndarray | None = None,
                      tight_mask: np.ndarray | None = None) -> dict:
    """folded.py:235-392 for a batch: board u8 [B,5] (255 = none), weights [B,P,H], status [B,P]."""

    batch, players, hands = range_weights.shape
    cards = 4 * ranks
    first_card = 52 - cards
    pair = combos(cards)
    folder_mask = status == FOLDED
    tight = folder_mask if tight_mask is None else tight_mask.astype(bool)
    raw = np.where(np.isfinite(range_weights), range_weights, 0.0).astype(np.float64)
    raw = np.maximum(raw, 0.0) * folder_mask[..., None]
    board_valid = board_cards != PAD_CARD
    global_pair = pair + first_card
    conflict = (board_valid[:, :, None, None] & (board_cards.astype(np.int64)[:, :, None, None] == global_pair[None, None])
                ).any(1).any(-1)                                             # [B,H]
    raw = np.where(conflict[:, None, :], 0.0, raw)
    mass = raw.sum(-1)
    probability = raw / np.maximum(mass, TINY)[..., None]
    base_cards = cards - board_valid.sum(-1)
    removal = removal_queries(cards)
    phi = np.zeros((batch, len(removal)))
    triple = np.zeros((batch, len(removal)))
    for b in range(batch):
        phi[b], triple[b] = phi_queries(probability[b], folder_mask[b], tight[b], float(base_cards[b]), removal)
    phi_zero = phi[:, :1]
    alpha = phi[:, 1: 1 + cards] - phi_zero
    pair_value = phi[:, 1 + cards:] - phi[:, 1 + pair[:, 0]] - phi[:, 1 + pair[:, 1]] + phi_zero
    beta = np.zeros((batch, cards, cards))
    beta[:, pair[:, 0], pair[:, 1]] = pair_value
    beta[:, pair[:, 1], pair[:, 0]] = pair_value
    # folded.py:330-336 scatters each board slot's validity at its clamped deck-local index, in slot
    # order, so an empty slot (255 clamps to the last card) written after the deck's last card clears
    # that card's mark; the sequential (CPU) order of that scatter is restated here
    on_board = np.zeros((batch, cards), dtype=bool)
    local = np.clip(board_cards.astype(np.int64) - first_card, 0, cards - 1)
    for slot in range(board_cards.shape[1]):
        on_board[np.arange(batch), local[:, slot]] = board_valid[:, slot]
    beta = np.where(on_board[:, :, None] | on_board[:, None, :], 0.0, beta)
    alpha = np.where(on_board, 0.0, alpha)
    hand_log_ratio = alpha[:, pair[:, 0]] + alpha[:, pair[:, 1]] + beta[:, pair[:, 0], pair[:, 1]]
    value, vector = np.linalg.eigh(beta)
    order = np.argsort(-np.abs(value), axis=-1, kind="stable")[:, :beta_rank]
    value = np.take_along_axis(value, order, 1)
    vector = np.take_along_axis(vector, order[:, None, :], 2)
    pivot = np.abs(vector).argmax(1)
    orientation = np.take_along_axis(vector, pivot[:, None, :], 1)[:, 0]
    vector = vector * np.where(orientation < 0, -1.0, 1.0)[:, None, :]
    incidence = np.zeros((hands, cards))
    incidence[np.arange(hands), pair[:, 0]] = 1.0
    incidence[np.arange(hands), pair[:, 1]] = 1.0
    line_dim = 0 if line_metadata is None else line_metadata.shape[-1]
    return {
        "phi": phi, "triple": triple, "beta": beta,
        "hand_log_ratio": hand_log_ratio,
        "beta_eigenvalue": value, "beta_eigenvector": vector,
        "folder_log_mass": np.where(folder_mask, np.log(np.maximum(mass, TINY)), 0.0),
        "folder_card_mass": raw @ incidence,
        "folder_line_meta": (np.zeros((batch, players, 0)) if line_metadata is None
                             else line_metadata * folder_mask[..., None]),
        "folder_mask": folder_mask,
        "folder_output_valid": folder_mask & (mass > 0),
        "folder_seat": np.broadcast_to(np.arange(players), (batch, players)),
        "tight_cluster_scalar": triple[:, 0],
        "line_dim": line_dim,
    }


def workspace_row_bytes(players: int, ranks: int) -> int:
    """folded.py:21-46: the reference's per-row admission bound for its folded-statistics workspace."""

    if players == 2:
        return 0
    cards = 4 * ranks
    hands = cards * (cards - 1) // 2
    queries = 1 + cards + hands
    chunk = min(queries, QUERY_CHUNK)
    values = (players * cards * cards + chunk * (2 * players * cards + players * players + 8 * players + 8)
              + 2 * queries + 10 * chunk * hands + hands + 3 * cards * cards)
    return 4 * values


def summary_width(players: int, ranks: int) -> int:
    """hooks.py:172-185 (NLHEGeometry.folded_summary_width)."""

    if players == 2:
        return 0
    cards = 4 * ranks
    return cards * (cards - 1) // 2 + cards + cards * cards + players + players * cards + 2


def family_workspace_row_bytes(players: int, ranks: int, base_input_width: int, m_raise: int) -> int:
    """folded.py:49-76 (sequential_family_workspace_row_bytes) given the postflop base input width."""

    cards = 4 * ranks
    hands = cards * (cards - 1) // 2
    width = base_input_width + summary_width(players, ranks)
    model = width + hands * (5 + 3 * m_raise)
    transition = 2 * width + 8 * players * hands + 4 * hands + 128 * players + 256
    return 4 * (model + transition) + workspace_row_bytes(players, ranks)


__all__ = ["combos", "family_workspace_row_bytes", "folded_statistics", "phi_queries", "removal_queries",
           "summary_width", "workspace_row_bytes"]
