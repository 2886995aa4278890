"""The folded-statistics restatement (oracle/folded_oracle.py) pinned by the reference itself.

tests/golden/folded.npz holds pbg/games/poker/queued/folded.py's own outputs (run on CPU by
tests/golden/make_golden.py): the per-query phi and triple terms recorded inside the call and the
returned summary, for 3-, 4- and 6-handed geometries (R4, R5, R13) with one to four folders, tight
subsets, flop/turn/river boards and ranges with zeros, negative and non-finite entries.  The
restatement computes in float64; the reference in float32, so the bars are float32 rounding bars
(phi 1e-5; Lambda_B 3e-5 as the reference's own finite-difference tests use).  The closed-form and
exact-enumeration checks restate tests/test_sequential_modes.py:556-755 of the reference.
"""

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import folded_oracle as fo  # noqa: E402

CASES = range(4)


def _case(d, i):
    p = f"c{i}_"
    players, _stack, ranks, beta_rank, _line = (int(x) for x in d[p + "geometry"])
    line = d[p + "line_metadata"] if p + "line_metadata" in d else None
    result = fo.folded_statistics(d[p + "board_cards"], d[p + "range_weights"].astype(np.float64), d[p + "status"],
                                  ranks, beta_rank, line, d[p + "tight_mask"])
    return p, result, ranks, beta_rank


@pytest.mark.parametrize("i", CASES)
def test_oracle_matches_reference_folded_statistics(gold, i):
    d = gold("folded")
    p, r, ranks, beta_rank = _case(d, i)
    np.testing.assert_allclose(r["phi"], d[p + "phi"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r["triple"], d[p + "triple"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(r["hand_log_ratio"], d[p + "hand_log_ratio"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(r["beta_eigenvalue"], d[p + "beta_eigenvalue"], rtol=1e-4, atol=5e-5)
    if beta_rank == 4 * ranks:  # full rank: the eigenpairs reconstruct beta
        vec, val = d[p + "beta_eigenvector"], d[p + "beta_eigenvalue"]
        np.testing.assert_allclose(np.einsum("bcr,br,bdr->bcd", vec, val, vec), r["beta"], atol=5e-5)
    np.testing.assert_allclose(r["folder_log_mass"], d[p + "folder_log_mass"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(r["folder_card_mass"], d[p + "folder_card_mass"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r["tight_cluster_scalar"], d[p + "tight_cluster_scalar"], rtol=1e-4, atol=1e-8)
    for name in ("folder_mask", "folder_output_valid", "folder_seat"):
        assert np.array_equal(r[name], d[p + name]), name
    np.testing.assert_allclose(r["folder_line_meta"], d[p + "folder_line_meta"])


def test_workspace_bounds_match_reference():
    # tests/test_sequential_modes.py:398-403 of the reference, plus the recorded per-case values
    assert fo.workspace_row_bytes(6, 13) == 3_691_536
    assert fo.summary_width(6, 13) == 4402
    assert fo.family_workspace_row_bytes(6, 13, 8 + 60 + 6 * 1326 + 10 * (128 * 6 + 18 - 128 + 1 + 3), 4) == 4_290_160


def test_workspace_bounds_match_recorded(gold):
    import importlib

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "ai-game-learning_b200"))
    folded = importlib.import_module("pbg_b200.folded")
    from pbg_b200.poker import NLHEGeometry

    d = gold("folded")
    geometries = [tuple(d[f"c{i}_geometry"][:3]) for i in CASES] + [(6, 128.0, 13)]
    for (players, stack, ranks), ws, fam in zip(geometries, d["workspace_row_bytes"], d["family_workspace_row_bytes"]):
        g = NLHEGeometry(int(players), float(stack), int(ranks))
        assert folded.folded_statistics_workspace_row_bytes(g) == ws == fo.workspace_row_bytes(int(players), int(ranks))
        assert folded.sequential_family_workspace_row_bytes(g, 4) == fam


def test_pack_and_unpack_round_trip(gold):
    import torch
    from pbg_b200.folded import pack_folded_statistics, unpack_folded_statistics
    from pbg_b200.poker import NLHEGeometry

    d = gold("folded")
    for i in (1, 2, 3):
        p = f"c{i}_"
        players, stack, ranks, beta_rank, _ = d[p + "geometry"]
        g = NLHEGeometry(int(players), float(stack), int(ranks))
        names = ("hand_log_ratio", "beta_eigenvalue", "beta_eigenvector", "folder_log_mass", "folder_card_mass",
                 "tight_cluster_scalar")
        summary = {n: torch.from_numpy(d[p + n]) for n in names}
        packed = pack_folded_statistics(g, summary)
        assert torch.equal(packed, torch.from_numpy(d[p + "packed"]))
        status = torch.from_numpy(d[p + "status"])
        line = torch.zeros((status.shape[0], int(players), 2))
        view = unpack_folded_statistics(g, packed, beta_rank=int(beta_rank), line_metadata=line, status=status)
        for n in names:
            assert torch.equal(view[n], summary[n]), n
        assert torch.equal(view["folder_mask"], status.eq(1))


def _empty_board(batch=1):
    return np.full((batch, 5), fo.PAD_CARD, dtype=np.uint8)


def test_one_folder_matches_closed_form():
    # reference tests/test_sequential_modes.py:556-608: one folder, alpha = log1p(-m), beta from pair survival
    ranks, cards = 4, 16
    pair = fo.combos(cards)
    hands = len(pair)
    raw = np.arange(1, hands + 1, dtype=np.float64)
    p = raw / raw.sum()
    weights = np.zeros((1, 2, hands))
    weights[0, 1] = raw
    status = np.array([[0, 1]])
    r = fo.folded_statistics(_empty_board(), weights, status, ranks, cards)
    marginal = np.zeros(cards)
    np.add.at(marginal, pair[:, 0], p)
    np.add.at(marginal, pair[:, 1], p)
    alpha = np.log1p(-marginal)
    survival = 1.0 - marginal[pair[:, 0]] - marginal[pair[:, 1]] + p
    pair_beta = np.log(survival) - alpha[pair[:, 0]] - alpha[pair[:, 1]]
    np.testing.assert_allclose(r["hand_log_ratio"][0], alpha[pair[:, 0]] + alpha[pair[:, 1]] + pair_beta,
                               atol=2e-5, rtol=2e-5)
    assert (r["beta_eigenvalue"] < 0).any() and (r["beta_eigenvalue"] > 0).any()


def test_two_folders_match_exact_enumeration():
    # reference tests/test_sequential_modes.py:611-662
    ranks, cards = 4, 16
    pair = fo.combos(cards)
    hands = len(pair)
    first = np.arange(1, hands + 1, dtype=np.float64)
    second = first[::-1].copy()
    weights = np.zeros((1, 3, hands))
    weights[0, 1], weights[0, 2] = first, second
    r = fo.folded_statistics(_empty_board(), weights, np.array([[0, 1, 1]]), ranks, cards)
    p = np.stack((first / first.sum(), second / second.sum()))
    disjoint = (pair[:, None, :, None] != pair[None, :, None, :]).all(-1).all(-1).astype(np.float64)
    base = p[0] @ disjoint @ p[1]
    for hand in range(0, hands, 17):
        survives = (pair != pair[hand][0]).all(-1) & (pair != pair[hand][1]).all(-1)
        part = (p[0] * survives) @ disjoint @ (p[1] * survives)
        np.testing.assert_allclose(r["hand_log_ratio"][0, hand], np.log(part / base), atol=3e-5, rtol=3e-5)


def test_three_loose_folders_calibrate_to_exact_enumeration():
    # reference tests/test_sequential_modes.py:706-755 (every folder tight, the default)
    ranks, cards = 4, 16
    pair = fo.combos(cards)
    hands = len(pair)
    ordinal = np.arange(hands, dtype=np.float64)
    p = np.stack([1.0 + 0.1 * np.sin(ordinal * (f + 1) * 0.07) for f in range(3)])
    p /= p.sum(-1, keepdims=True)
    weights = np.zeros((1, 4, hands))
    weights[0, 1:] = p
    status = np.array([[0, 1, 1, 1]])
    r = fo.folded_statistics(_empty_board(), weights, status, ranks, cards)
    disjoint = (pair[:, None, :, None] != pair[None, :, None, :]).all(-1).all(-1).astype(np.float64)

    def exact(w):
        return np.einsum("h,i,j,hi,hj,ij->", w[0], w[1], w[2], disjoint, disjoint, disjoint)

    base = exact(p)
    for hand in range(0, hands, 17):
        survives = (pair != pair[hand][0]).all(-1) & (pair != pair[hand][1]).all(-1)
        np.testing.assert_allclose(r["hand_log_ratio"][0, hand], np.log(exact(p * survives) / base),
                                   atol=1e-3, rtol=1e-3)
