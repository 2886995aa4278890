"""CPU checks of the Rao-Blackwell completion estimator (oracle restatement).

The external evaluator's ``complete`` / ``complete_selected`` (called at
pbg/games/poker/queued/hooks.py:2472-2477, 2512) is not in the reference tree,
so parity with it is unpinned.  What these tests pin instead is the law it
estimates, PreTerminalMC (docs/theory/core_math.tex:664-684): on small decks
the exact posterior of each seat's hand, P(x) ∝ Π_q w_q(x_q) over card-disjoint
profiles, and the exact conditional mean return are enumerated here, and the
oracle's importance-sampled estimates must converge to them.  The device
kernel is checked bit for bit against this oracle in test_gpu_completion.py.
"""

from __future__ import annotations

import itertools
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as O  # noqa: E402

PAD = 255


def _hands(D: int):
    return [(a, b) for a in range(D) for b in range(a + 1, D)]


def exact_completion(rank_count, board, weights, level, base, amount):
    """Exact p[P,H] and v[P,H] of one leaf row by enumeration (profiles x board runouts)."""

    D = 4 * rank_count
    first = 52 - D
    hands = _hands(D)
    P, H = weights.shape
    known = [c - first for c in board if c != PAD]
    missing = 5 - len(known)
    legal = [h for h, (a, b) in enumerate(hands) if a not in known and b not in known]
    per_seat = [[h for h in legal if weights[q, h] > 0] for q in range(P)]
    profiles, masses = [], []
    for prof in itertools.product(*per_seat):
        cards = [c for h in prof for c in hands[h]]
        if len(set(cards)) != len(cards):
            continue
        profiles.append(prof)
        masses.append(np.prod([float(weights[q, h]) for q, h in enumerate(prof)]))
    masses = np.array(masses) / np.sum(masses)
    rows_board, rows_combo, owner = [], [], []
    for k, prof in enumerate(profiles):
        used = set(known) | {c for h in prof for c in hands[h]}
        rest = [c for c in range(D) if c not in used]
        for runout in itertools.combinations(rest, missing):
            full = [c for c in board if c != PAD] + [c + first for c in runout]
            rows_board.append(full)
            rows_combo.append(prof)
            owner.append(k)
    owner = np.array(owner)
    B = len(owner)
    payoff = O.evaluate_showdowns(rank_count, np.array(rows_board, np.uint8), np.array(rows_combo, np.int32),
                                  np.broadcast_to(level, (B, P)), np.broadcast_to(base, (B, P)),
                                  np.broadcast_to(amount, (B, amount.size)))
    count = np.bincount(owner, minlength=len(profiles)).astype(np.float64)
    mean_payoff = np.zeros((len(profiles), P))
    np.add.at(mean_payoff, owner, payoff.astype(np.float64))
    mean_payoff /= count[:, None]
    p = np.zeros((P, H))
    pv = np.zeros((P, H))
    for k, prof in enumerate(profiles):
        for q, h in enumerate(prof):
            p[q, h] += masses[k]
            pv[q, h] += masses[k] * mean_payoff[k, q]
    variance = np.zeros(P)
    ev = (masses[:, None] * mean_payoff).sum(0)
    for q in range(P):  # variance of a single sampled return (profile and runout)
        variance[q] = np.sum(masses[owner] / count[owner] * (payoff[:, q] - ev[q]) ** 2)
    v = np.divide(pv, p, out=np.zeros_like(pv), where=p > 0)
    return p, v, ev, variance


def _row(rank_count, P, board, seed, concentrated=False):
    D = 4 * rank_count
    H = D * (D - 1) // 2
    rng = np.random.default_rng(seed)
    w = rng.random((P, H)).astype(np.float32)
    w[rng.random((P, H)) < 0.3] = 0.0
    if concentrated:  # every seat leans on the same few high cards: many proposal collisions
        hands = _hands(D)
        for h, (a, b) in enumerate(hands):
            if a >= D - 4 or b >= D - 4:
                w[:, h] *= 200.0
    level = np.ones(P, np.int32)
    level[-1] = 0  # the last seat contests only the first stratum
    base = -np.arange(1, P + 1, dtype=np.float32)
    amount = np.zeros(P, np.float32)
    amount[0] = float(P)
    amount[1] = float(np.sum(np.arange(1, P + 1)) - P)
    return np.array(board, np.uint8), w, level, base, amount


@pytest.mark.parametrize("case", [
    (4, 2, [36, 41, 46, 51, 40], False),     # river, heads-up
    (4, 2, [36, 41, 46, 51, PAD], False),    # turn: one runout card
    (4, 2, [36, 41, 46, 51, PAD], True),     # concentrated ranges
    (4, 3, [36, 41, 46, 51, 40], False),     # river, three seats
])
def test_estimator_converges_to_exact_enumeration(case):
    R, P, board, concentrated = case
    board, w, level, base, amount = _row(R, P, board, 7, concentrated)
    p, v, ev, var = exact_completion(R, board, w, level, base, amount)
    N = 20000
    ph, vh, ne, status = O.rb_complete(R, board[None], w[None], level[None], base[None], amount[None], N,
                                       np.array([11]))
    assert status == 0
    ph, vh, ne = ph[0].astype(np.float64), vh[0].astype(np.float64), float(ne[0])
    assert 0 < ne <= N
    np.testing.assert_allclose(ph.sum(-1), 1.0, rtol=0, atol=2e-6)
    # chi-square of every seat's hand occurrence against the exact posterior
    for q in range(P):
        live = p[q] > 0
        assert np.all(ph[q][~live] == 0)
        stat = np.sum((ph[q][live] - p[q][live]) ** 2 / (p[q][live] / ne))
        dof = live.sum() - 1
        assert stat < dof + 8 * np.sqrt(2 * dof), (q, stat, dof)
        # seat value: sum_h p_hat v_hat against the exact expectation
        est = float(np.sum(ph[q] * vh[q]))
        assert abs(est - ev[q]) < 6 * np.sqrt(var[q] / ne) + 1e-6, (q, est, ev[q])
    # conditional values of the likeliest hands of seat 0
    top = np.argsort(-p[0])[:5]
    for h in top:
        sd = np.sqrt(var[0] / max(ne * p[0, h], 1.0)) * 2.0
        assert abs(vh[0, h] - v[0, h]) < 6 * sd + 1e-6


def test_chips_are_conserved_and_selected_equals_dense():
    R, P = 13, 6
    D = 52
    H = D * (D - 1) // 2
    rng = np.random.default_rng(3)
    F = 4
    board = np.full((F, 5), PAD, np.uint8)
    board[1, :3] = [0, 17, 33]
    board[2, :4] = [5, 9, 44, 50]
    board[3] = [2, 7, 12, 30, 48]
    w = np.exp(rng.normal(0, 2, (F, P, H))).astype(np.float32)
    level = np.tile(np.array([2, 0, 1, -1, 2, 0], np.int32), (F, 1))
    base = -rng.integers(1, 20, (F, P)).astype(np.float32)
    base[:, 3] = -1.0
    amount = np.zeros((F, 3), np.float32)
    amount[:, 0] = 10.0
    pot = -base.sum(1)
    amount[:, 1] = (pot - 10.0) / 2
    amount[:, 2] = pot - 10.0 - amount[:, 1]
    seed = np.array([5, 6, 7, 8], np.int64)
    ph, vh, ne, status = O.rb_complete(R, board, w, level, base, amount, 300, seed)
    assert status == 0 and np.all(ne > 0) and np.all(ne <= 300)
    totals = (ph.astype(np.float64) * vh).sum(-1).sum(-1)  # sum over seats of the seat values
    np.testing.assert_allclose(totals, 0.0, atol=2e-3)
    sel = np.array([0, 3, 5, 2], np.int32)
    sp, sv, sn, sstatus = O.rb_complete(R, board, w, level, base, amount, 300, seed, selected_player=sel)
    assert sstatus == 0
    np.testing.assert_array_equal(sp, ph[np.arange(F), sel])
    np.testing.assert_array_equal(sv, vh[np.arange(F), sel])
    np.testing.assert_array_equal(sn, ne)
    again = O.rb_complete(R, board, w, level, base, amount, 300, seed)
    np.testing.assert_array_equal(again[0], ph)
    other = O.rb_complete(R, board, w, level, base, amount, 300, seed + 1)
    assert not np.array_equal(other[0], ph)


def test_uniform_heads_up_ranges_have_full_effective_size():
    R, P = 4, 2
    H = 120
    w = np.ones((1, P, H), np.float32)
    board = np.full((1, 5), PAD, np.uint8)
    level = np.zeros((1, P), np.int32)
    base = np.full((1, P), -3.0, np.float32)
    amount = np.array([[6.0, 0.0]], np.float32)
    ph, vh, ne, status = O.rb_complete(R, board, w, level, base, amount, 1000, np.array([1]))
    assert status == 0
    assert ne[0] == np.float32(1000)


def test_rows_without_mass_and_invalid_rows_are_flagged():
    R, P = 4, 2
    H = 120
    w = np.ones((3, P, H), np.float32)
    w[0, 1] = 0.0  # seat 1 has no weight
    board = np.full((3, 5), PAD, np.uint8)
    board[1, 0] = 3  # not a card of the 16-card deck
    board[2, :2] = [40, 40]  # repeated card
    level = np.zeros((3, P), np.int32)
    base = np.zeros((3, P), np.float32)
    amount = np.ones((3, 1), np.float32)
    ph, vh, ne, status = O.rb_complete(R, board, w, level, base, amount, 8, np.arange(3))
    assert status == 3
    assert np.all(ne == 0) and np.all(ph == 0) and np.all(vh == 0)
