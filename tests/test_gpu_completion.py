"""Rao-Blackwell leaf completion (contract-v2 ``complete`` / ``complete_selected``) on the GPU.

The external evaluator that the reference calls at
pbg/games/poker/queued/hooks.py:2472-2477, 2512 is not in the reference tree:
parity with it is unpinned.  The device estimator must equal the C restatement
(oracle ``rb_complete``) bit for bit -- p_hat, v_hat and n_eff -- on seeded
leaves of every board street, folded seats, concentrated ranges (collisions
and exact scans) and sample counts that do not fill the thread block; the
oracle itself converges to the exact enumerated law (test_completion_oracle.py),
checked here once more on the device at a large sample count.  The selected
variant equals the dense slice exactly, as the reference's own test
(tests/test_sequential_modes.py:666-696) requires.
"""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
PAD = 255


def _leaves(R, P, F, seed, concentrated=False):
    D = 4 * R
    H = D * (D - 1) // 2
    first = 52 - D
    rng = np.random.default_rng(seed)
    board = np.full((F, 5), PAD, np.uint8)
    for f in range(F):
        shown = [0, 3, 4, 5][f % 4]
        board[f, :shown] = rng.permutation(D)[:shown] + first
    w = np.exp(rng.normal(0.0, 1.5, (F, P, H))).astype(np.float32)
    w[rng.random(w.shape) < 0.2] = 0.0
    if concentrated:  # every seat leans on the four top cards
        a, b = np.triu_indices(D, 1)
        top = (a >= D - 4) | (b >= D - 4)
        w[:, :, top] *= 500.0
    level = rng.integers(-1, 3, (F, P)).astype(np.int32)
    level[:, 0] = np.maximum(level[:, 0], 0)
    level[:, 1] = np.maximum(level[:, 1], 0)
    base = -rng.integers(1, 30, (F, P)).astype(np.float32) * 0.5
    pot = -base.sum(1)
    amount = np.stack([pot * 0.5, pot * 0.3, pot * 0.2], 1).astype(np.float32)
    seed_col = rng.integers(-2**62, 2**62, F, dtype=np.int64)
    return board, w, level, base, amount, seed_col


def _device(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in arrays]


def _evaluator(R):
    import poker_gpu_evaluator as E

    return E.bind(rank_count=R)


@pytest.mark.parametrize("R,P,F,N,concentrated", [
    (4, 2, 8, 64, False), (4, 2, 8, 257, True), (4, 3, 6, 4, False), (6, 3, 5, 700, True),
    (13, 2, 6, 2000, False), (13, 6, 6, 300, False), (13, 6, 4, 1024, True),
])
def test_completion_matches_oracle(R, P, F, N, concentrated):
    board, w, level, base, amount, seed = _leaves(R, P, F, R * 100 + P * 10 + N, concentrated)
    ev = _evaluator(R)
    tb, tw, tl, tbase, tamt, tseed = _device(board, w, level, base, amount, seed)
    common = dict(board_cards=tb, range_weights=tw, stratum_level=tl, payoff_baseline=tbase, stratum_amount=tamt,
                  n_samples=N, seed=tseed)
    dense = ev.complete(**common)
    ph, vh, ne, status = O.rb_complete(R, board, w, level, base, amount, N, seed)
    assert status == 0
    assert np.array_equal(dense.p_hat.cpu().numpy(), ph)
    assert np.array_equal(dense.v_hat.cpu().numpy(), vh)
    assert np.array_equal(dense.n_eff.cpu().numpy(), ne)
    assert bool((dense.n_eff > 0).all()) and bool((dense.n_eff <= N + 1e-4).all())
    sel = np.random.default_rng(N).integers(0, P, F).astype(np.int32)
    compact = ev.complete_selected(**common, selected_player=torch.from_numpy(sel).to(DEV))
    rows = torch.arange(F, device=DEV)
    tsel = torch.from_numpy(sel).long().to(DEV)
    assert torch.equal(compact.p_hat, dense.p_hat[rows, tsel])
    assert torch.equal(compact.v_hat, dense.v_hat[rows, tsel])
    assert torch.equal(compact.n_eff, dense.n_eff)


def test_completion_rows_are_independent_of_batching():
    R, P, F, N = 13, 6, 24, 256
    board, w, level, base, amount, seed = _leaves(R, P, F, 5)
    ev = _evaluator(R)
    full = ev.complete(**dict(zip(("board_cards", "range_weights", "stratum_level", "payoff_baseline",
                                   "stratum_amount", "seed"), _device(board, w, level, base, amount, seed))),
                       n_samples=N)
    pick = np.arange(3, F, 5)
    part = ev.complete(**dict(zip(("board_cards", "range_weights", "stratum_level", "payoff_baseline",
                                   "stratum_amount", "seed"),
                                  _device(board[pick], w[pick], level[pick], base[pick], amount[pick], seed[pick]))),
                       n_samples=N)
    idx = torch.from_numpy(pick).to(DEV)
    assert torch.equal(part.p_hat, full.p_hat[idx])
    assert torch.equal(part.v_hat, full.v_hat[idx])


def test_device_estimator_converges_to_exact_law():
    import test_completion_oracle as T

    R, P = 4, 2
    board, w, level, base, amount = T._row(R, P, [36, 41, 46, 51, PAD], 7, True)
    p, v, expected, var = T.exact_completion(R, board, w, level, base, amount)
    ev = _evaluator(R)
    N = ev.max_samples(P)
    tb, tw, tl, tbase, tamt = _device(board[None], w[None], level[None], base[None], amount[None])
    out = ev.complete(board_cards=tb, range_weights=tw, stratum_level=tl, payoff_baseline=tbase, stratum_amount=tamt,
                      n_samples=N, seed=torch.tensor([3], device=DEV))
    ph = out.p_hat[0].double().cpu().numpy()
    vh = out.v_hat[0].double().cpu().numpy()
    ne = float(out.n_eff[0])
    for q in range(P):
        live = p[q] > 0
        stat = np.sum((ph[q][live] - p[q][live]) ** 2 / (p[q][live] / ne))
        dof = live.sum() - 1
        assert stat < dof + 8 * np.sqrt(2 * dof)
        assert abs(np.sum(ph[q] * vh[q]) - expected[q]) < 6 * np.sqrt(var[q] / ne)


def test_rb_leaf_then_selected_completion_matches_dense_slice():
    """The reference's tests/test_sequential_modes.py:666-696 on this build's state machine and evaluator."""

    from pbg_b200.poker import NLHEGeometry, PokerStateMachine

    geometry = NLHEGeometry(3, 8.0, 4)
    machine = PokerStateMachine(geometry)
    state = machine.initial_roots(1, seed=43, iteration=0, retry_epoch=0, device=DEV)
    leaf = machine.rb_leaf(state, torch.zeros((1, 3, geometry.private_hands), dtype=torch.float32, device=DEV),
                           seed=torch.tensor([71], dtype=torch.int64, device=DEV))
    common = {"board_cards": leaf["leaf_public_state"], "range_weights": leaf["range_weights"],
              "stratum_level": leaf["stratum_level"], "payoff_baseline": leaf["payoff_baseline"],
              "stratum_amount": leaf["stratum_amount"], "n_samples": 4, "seed": leaf["seed"]}
    ev = _evaluator(geometry.rank_count)
    dense = ev.complete(**common)
    compact = ev.complete_selected(**common, selected_player=torch.tensor([1], dtype=torch.int32, device=DEV))
    torch.testing.assert_close(compact.p_hat, dense.p_hat[:, 1], rtol=0, atol=0)
    torch.testing.assert_close(compact.v_hat, dense.v_hat[:, 1], rtol=0, atol=0)
    host = {k: (v.cpu().numpy() if isinstance(v, torch.Tensor) else v) for k, v in common.items()}
    ph, vh, ne, status = O.rb_complete(4, host["board_cards"], host["range_weights"], host["stratum_level"],
                                       host["payoff_baseline"], host["stratum_amount"], 4, host["seed"])
    assert status == 0
    assert np.array_equal(dense.p_hat.cpu().numpy(), ph) and np.array_equal(dense.v_hat.cpu().numpy(), vh)


def test_rb_leaf_range_weights():
    from pbg_b200.poker import NLHEGeometry, PokerStateMachine

    geometry = NLHEGeometry(2, 100.0, 13)
    machine = PokerStateMachine(geometry)
    state = machine.initial_roots(4, seed=3, iteration=0, retry_epoch=0, device=DEV)
    g = torch.Generator().manual_seed(1)
    reach = torch.randn((4, 2, geometry.private_hands), generator=g) * 5
    reach[0, 0, :10] = -torch.inf
    reach[1, 1, :] = -torch.inf  # a seat that cannot be here: all weights 0
    reach[2, 0, 7] = torch.nan
    leaf = machine.rb_leaf(state, reach.to(DEV), seed=torch.arange(4, device=DEV),
                           selected_player=torch.tensor([0, 1, 0, 1], device=DEV))
    w = leaf["range_weights"]
    reach = reach.to(DEV)  # hooks.py:1238-1242, written as the reference writes it
    finite = torch.isfinite(reach)
    gauge = reach.masked_fill(~finite, -torch.inf).amax(-1, keepdim=True)
    expect = torch.exp(reach - gauge.masked_fill(~torch.isfinite(gauge), 0.0)).masked_fill(~finite, 0.0)
    assert torch.equal(w, expect)
    assert float(w[1, 1].sum()) == 0.0
    assert leaf["trained_actor"].dtype == torch.int32
    assert torch.equal(leaf["leaf_public_state"], state.board_cards)
    assert leaf["stratum_amount"].shape == (4, 2) and leaf["seed"].dtype == torch.int64


def test_completion_flags_rows_it_cannot_estimate():
    import poker_gpu_evaluator as E

    R, P = 4, 2
    board, w, level, base, amount, seed = _leaves(R, P, 3, 1)
    ev = _evaluator(R)
    w0 = w.copy()
    w0[1, 1] = 0.0
    args = dict(zip(("board_cards", "range_weights", "stratum_level", "payoff_baseline", "stratum_amount", "seed"),
                    _device(board, w0, level, base, amount, seed)))
    with pytest.raises(E.EvaluatorError):
        ev.complete(**args, n_samples=16)
    out = ev.complete(**args, n_samples=16, validate=False)
    assert float(out.n_eff[1]) == 0.0 and float(out.p_hat[1].abs().sum()) == 0.0
    bad = board.copy()
    bad[0, :2] = [40, 40]
    args = dict(zip(("board_cards", "range_weights", "stratum_level", "payoff_baseline", "stratum_amount", "seed"),
                    _device(bad, w, level, base, amount, seed)))
    with pytest.raises(ValueError):
        ev.complete(**args, n_samples=16)
    with pytest.raises(ValueError):
        ev.complete_selected(**dict(args, board_cards=_device(board)[0]), n_samples=16,
                             selected_player=torch.tensor([0, 2, 1], dtype=torch.int32, device=DEV))
    from pbg_b200._native import NativeError

    with pytest.raises((ValueError, NativeError)):
        ev.complete(**dict(args, board_cards=_device(board)[0]), n_samples=ev.max_samples(P) + 1)
