"""Contract-v2 poker evaluator binding backed by libpbgb200 (sm_100a).

pbg loads its showdown evaluator through
pbg/games/poker/queued/evaluator.py:9-35 (``CONTRACT_VERSION == "2"``,
``bind(rank_count=...)``, ``info.contract_version``/``info.rank_count``) and
calls ``evaluate_showdowns(board_cards=, combo_ids=, stratum_level=,
payoff_baseline=, stratum_amount=)`` at hooks.py:2277-2295.  This module
provides exactly that surface; ranking follows standard 7-card NLHE with
the rarity-consistent short-deck category order of pbg's cards.py:37-74.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass

import torch

_HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

from pbg_b200._native import call, ptr, stream  # noqa: E402

CONTRACT_VERSION = "2"


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


def bind(rank_count: int) -> BoundEvaluator:
    return BoundEvaluator(rank_count)
