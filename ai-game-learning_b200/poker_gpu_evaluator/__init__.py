"""Contract-v2 poker evaluator binding backed by libpbgb200 (sm_100a).

pbg loads its showdown evaluator through
pbg/games/poker/queued/evaluator.py:9-35 (``CONTRACT_VERSION == "2"``,
``bind(rank_count=...)``, ``info.contract_version``/``info.rank_count``) and
calls ``evaluate_showdowns(board_cards=, combo_ids=, stratum_level=,
payoff_baseline=, stratum_amount=)`` at hooks.py:2277-2295 and, for
Rao-Blackwell leaves, ``complete(board_cards=, range_weights=,
stratum_level=, payoff_baseline=, stratum_amount=, n_samples=, seed=)`` /
``complete_selected(..., selected_player=)`` at hooks.py:2472-2477, 2512,
reading ``.p_hat``, ``.v_hat`` and ``.n_eff`` of the result.  This module
provides exactly that surface; ranking follows standard 7-card NLHE with
the rarity-consistent short-deck category order of pbg's cards.py:37-74, and
completion is the PreTerminalMC law of the reference's theory
(docs/theory/core_math.tex:664-684) estimated by libpbgb200's
``pbg_rb_complete``.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass

import torch

_HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

from pbg_b200 import _native as N  # noqa: E402
from pbg_b200._native import call, ptr, stream  # noqa: E402

CONTRACT_VERSION = "2"


class EvaluatorError(RuntimeError):
    """A completion row that cannot be estimated (a seat without board-legal range weight)."""


@dataclass(frozen=True)
class Completion:
    """p_hat / v_hat f32 [F,P,H] from ``complete`` ([F,H] from ``complete_selected``), n_eff f32 [F]."""

    p_hat: torch.Tensor
    v_hat: torch.Tensor
    n_eff: torch.Tensor


@dataclass(frozen=True)
class EvaluatorInfo:
    contract_version: str
    rank_count: int


class BoundEvaluator:
    def __init__(self, rank_count: int) -> None:
        if isinstance(rank_count, bool) or not isinstance(rank_count, int) or not 4 <= rank_count <= 13:
            raise ValueError("rank_count must be an integer in [4,13]")
        self.info = EvaluatorInfo(CONTRACT_VERSION, rank_count)

    def evaluate_showdowns(self, *, board_cards, combo_ids, stratum_level, payoff_baseline, stratum_amount):
        B, P = combo_ids.shape
        if board_cards.shape != (B, 5) or stratum_level.shape != (B, P) or payoff_baseline.shape != (B, P) \
                or stratum_amount.ndim != 2 or stratum_amount.shape[0] != B:
            raise ValueError("evaluate_showdowns: inconsistent shapes")
        out = torch.empty((B, P), dtype=torch.float32, device=combo_ids.device)
        call("pbg_evaluate_showdowns", self.info.rank_count, B, P, stratum_amount.shape[1],
             ptr(board_cards.to(torch.uint8).contiguous()), ptr(combo_ids.to(torch.int32).contiguous()),
             ptr(stratum_level.to(torch.int32).contiguous()), ptr(payoff_baseline.float().contiguous()),
             ptr(stratum_amount.float().contiguous()), ptr(out), stream(combo_ids.device))
        return out


    def max_samples(self, players: int) -> int:
        """Largest ``n_samples`` one completion call accepts for ``players`` seats."""

        return int(N.lib().pbg_rb_complete_max_samples(self.info.rank_count, int(players)))

    def complete(self, *, board_cards, range_weights, stratum_level, payoff_baseline, stratum_amount, n_samples,
                 seed, validate: bool = True) -> Completion:
        """Every seat's completion of each Rao-Blackwell leaf row: p_hat, v_hat [F,P,H]."""

        return self._complete(board_cards, range_weights, stratum_level, payoff_baseline, stratum_amount, n_samples,
                              seed, None, validate)

    def complete_selected(self, *, board_cards, range_weights, stratum_level, payoff_baseline, stratum_amount,
                          n_samples, seed, selected_player, validate: bool = True) -> Completion:
        """The selected seat's completion of each row: p_hat, v_hat [F,H], bit-identical to
        ``complete(...).p_hat[f, selected_player[f]]``."""

        return self._complete(board_cards, range_weights, stratum_level, payoff_baseline, stratum_amount, n_samples,
                              seed, selected_player, validate)

    def _complete(self, board_cards, range_weights, stratum_level, payoff_baseline, stratum_amount, n_samples, seed,
                  selected_player, validate):
        if range_weights.ndim != 3:
            raise ValueError("complete: range_weights must be [F,P,H]")
        F, P, H = range_weights.shape
        D = 4 * self.info.rank_count
        if H != D * (D - 1) // 2:
            raise ValueError(f"complete: {H} private hands do not match a {D}-card deck")
        if (board_cards.shape != (F, 5) or stratum_level.shape != (F, P) or payoff_baseline.shape != (F, P)
                or stratum_amount.ndim != 2 or stratum_amount.shape[0] != F or seed.numel() != F
                or (selected_player is not None and selected_player.numel() != F)):
            raise ValueError("complete: inconsistent shapes")
        if isinstance(n_samples, bool) or int(n_samples) != n_samples or n_samples <= 0:
            raise ValueError("complete: n_samples must be a positive integer")
        dev = range_weights.device
        out_shape = (F, P, H) if selected_player is None else (F, H)
        p_hat = torch.empty(out_shape, dtype=torch.float32, device=dev)
        v_hat = torch.empty(out_shape, dtype=torch.float32, device=dev)
        n_eff = torch.empty(F, dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        sel = None if selected_player is None else selected_player.to(torch.int32).reshape(F).contiguous()
        call("pbg_rb_complete", self.info.rank_count, F, P, stratum_amount.shape[1], int(n_samples),
             ptr(board_cards.to(torch.uint8).contiguous()), ptr(range_weights.float().contiguous()),
             ptr(stratum_level.to(torch.int32).contiguous()), ptr(payoff_baseline.float().contiguous()),
             ptr(stratum_amount.float().contiguous()), ptr(seed.to(torch.int64).reshape(F).contiguous()), ptr(sel),
             ptr(p_hat), ptr(v_hat), ptr(n_eff), ptr(status), stream(dev))
        if validate and F:
            code = int(status.item())
            if code & 1:
                raise ValueError("complete: a row has an invalid board card or selected seat")
            if code & 2:
                raise EvaluatorError("complete: a row has no sample mass (a seat without board-legal range weight)")
        return Completion(p_hat, v_hat, n_eff)


def bind(rank_count: int) -> BoundEvaluator:
    return BoundEvaluator(rank_count)
