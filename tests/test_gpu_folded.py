"""pbg_folded_phi_queries and pbg_b200.folded.folded_statistics on the GPU against the reference.

Goldens: tests/golden/folded.npz, the reference's own float32 outputs (CPU run).  Bars are the
float32 rounding bars of the CPU tests (phi 1e-5 absolute; Lambda_B 3e-5, the reference's own
finite-difference test bar); the restatement oracle/folded_oracle.py (float64) checks larger random
6-handed R13 batches.  The closed-form and exact-enumeration tests restate the reference's
tests/test_sequential_modes.py:556-755 on this build's kernel.
"""

import os
import sys
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import folded_oracle as fo  # noqa: E402


def _machine(players, stack, ranks):
    from pbg_b200.poker import NLHEGeometry, PokerStateMachine

    geometry = NLHEGeometry(players, stack, ranks)
    machine = PokerStateMachine(geometry)
    combo = machine.combo_cards(torch.arange(geometry.private_hands, dtype=torch.int32, device=DEV))
    return geometry, combo


def _run(d, i):
    from pbg_b200.folded import folded_statistics

    p = f"c{i}_"
    players, stack, ranks, beta_rank, line_dim = d[p + "geometry"]
    geometry, combo = _machine(int(players), float(stack), int(ranks))
    line = torch.from_numpy(d[p + "line_metadata"]).to(DEV) if p + "line_metadata" in d else None
    return folded_statistics(geometry, board_cards=torch.from_numpy(d[p + "board_cards"]).to(DEV),
                             range_weights=torch.from_numpy(d[p + "range_weights"]).to(DEV),
                             status=torch.from_numpy(d[p + "status"]).to(DEV), combo_cards=combo,
                             beta_rank=int(beta_rank), line_dim=int(line_dim), line_metadata=line,
                             tight_mask=torch.from_numpy(d[p + "tight_mask"]).to(DEV)), p, int(ranks), int(beta_rank)


def _probability(weights, status, board, first_card, combo):
    folder = status.eq(1)
    raw = weights.masked_fill(~torch.isfinite(weights), 0.0).clamp_min(0.0) * folder[..., None]
    valid = board.ne(255)
    conflict = (valid[..., None, None] & board.long()[..., None, None].eq(combo[None])).any(1).any(-1)
    raw = raw.masked_fill(conflict[:, None], 0.0)
    prob = raw / raw.sum(-1).clamp_min(torch.finfo(torch.float32).tiny)[..., None]
    return prob, folder, valid


@pytest.mark.parametrize("i", range(4))
def test_phi_queries_match_reference(gold, i):
    from pbg_b200.folded import phi_queries

    d = gold("folded")
    p = f"c{i}_"
    players, stack, ranks, _, _ = d[p + "geometry"]
    geometry, combo = _machine(int(players), float(stack), int(ranks))
    board = torch.from_numpy(d[p + "board_cards"]).to(DEV)
    prob, folder, valid = _probability(torch.from_numpy(d[p + "range_weights"]).to(DEV),
                                       torch.from_numpy(d[p + "status"]).to(DEV), board, geometry.first_card, combo)
    base = geometry.deck_cards - valid.sum(-1, dtype=torch.float32)
    phi, triple = phi_queries(prob, folder, torch.from_numpy(d[p + "tight_mask"]).to(DEV), base, geometry.deck_cards)
    torch.cuda.synchronize()
    print(f"\ncase {i}: max |phi - reference| {float((phi.cpu() - torch.from_numpy(d[p + 'phi'])).abs().max()):.2e}")
    np.testing.assert_allclose(phi.cpu().numpy(), d[p + "phi"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(triple.cpu().numpy(), d[p + "triple"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("i", range(4))
def test_folded_statistics_match_reference(gold, i):
    d = gold("folded")
    r, p, ranks, beta_rank = _run(d, i)
    got = {k: v.cpu().numpy() for k, v in r.items()}
    np.testing.assert_allclose(got["hand_log_ratio"], d[p + "hand_log_ratio"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(got["beta_eigenvalue"], d[p + "beta_eigenvalue"], rtol=1e-4, atol=5e-5)
    if beta_rank == 4 * ranks:
        def rec(vec, val):
            return np.einsum("bcr,br,bdr->bcd", vec, val, vec)

        np.testing.assert_allclose(rec(got["beta_eigenvector"], got["beta_eigenvalue"]),
                                   rec(d[p + "beta_eigenvector"], d[p + "beta_eigenvalue"]), atol=5e-5)
    np.testing.assert_allclose(got["folder_log_mass"], d[p + "folder_log_mass"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got["folder_card_mass"], d[p + "folder_card_mass"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got["tight_cluster_scalar"], d[p + "tight_cluster_scalar"], rtol=1e-4, atol=1e-8)
    np.testing.assert_allclose(got["folder_line_meta"], d[p + "folder_line_meta"])
    for name in ("folder_mask", "folder_output_valid", "folder_seat"):
        assert np.array_equal(got[name], d[p + name]), name


def test_deterministic_and_matches_oracle_six_handed_full_deck():
    from pbg_b200.folded import folded_statistics

    geometry, combo = _machine(6, 100.0, 13)
    g = torch.Generator(device=DEV).manual_seed(77)
    batch = 3
    status = torch.zeros((batch, 6), dtype=torch.int8, device=DEV)
    status[0, [1, 2, 4]] = 1
    status[1, [0, 1, 2, 3]] = 1
    status[2, [5, 3]] = 1
    tight = status.eq(1).clone()
    tight[1, 2] = False
    board = torch.full((batch, 5), 255, dtype=torch.uint8, device=DEV)
    board[0, :3] = torch.tensor([3, 17, 40], dtype=torch.uint8)
    board[1, :4] = torch.tensor([51, 0, 22, 9], dtype=torch.uint8)
    board[2, :5] = torch.tensor([5, 6, 7, 8, 50], dtype=torch.uint8)
    weights = torch.rand((batch, 6, 1326), generator=g, device=DEV)
    args = dict(board_cards=board, range_weights=weights, status=status, combo_cards=combo, beta_rank=52, line_dim=0,
                tight_mask=tight)
    first = folded_statistics(geometry, **args)
    second = folded_statistics(geometry, **args)
    for name in first:
        assert torch.equal(first[name], second[name]), name
    want = fo.folded_statistics(board.cpu().numpy(), weights.cpu().numpy().astype(np.float64),
                                status.cpu().numpy(), 13, 52, None, tight.cpu().numpy())
    np.testing.assert_allclose(first["hand_log_ratio"].cpu().numpy(), want["hand_log_ratio"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(first["tight_cluster_scalar"].cpu().numpy(), want["tight_cluster_scalar"],
                               rtol=1e-4, atol=1e-8)


def test_one_folder_matches_closed_form():
    from pbg_b200.folded import folded_statistics

    geometry, combo = _machine(2, 8.0, 4)
    local = (combo - geometry.first_card).long()
    raw = torch.arange(1, geometry.private_hands + 1, dtype=torch.float32, device=DEV)
    p = raw / raw.sum()
    ranges = torch.zeros((1, 2, geometry.private_hands), device=DEV)
    ranges[0, 1] = raw
    status = torch.tensor([[0, 1]], dtype=torch.int8, device=DEV)
    board = torch.full((1, 5), 255, dtype=torch.uint8, device=DEV)
    r = folded_statistics(geometry, board_cards=board, range_weights=ranges, status=status, combo_cards=combo,
                          beta_rank=geometry.deck_cards, line_dim=0)
    marginal = torch.zeros(geometry.deck_cards, device=DEV)
    marginal.scatter_add_(0, local[:, 0], p)
    marginal.scatter_add_(0, local[:, 1], p)
    alpha = torch.log1p(-marginal)
    survival = 1.0 - marginal[local[:, 0]] - marginal[local[:, 1]] + p
    pair_beta = torch.log(survival) - alpha[local[:, 0]] - alpha[local[:, 1]]
    beta = torch.zeros((geometry.deck_cards, geometry.deck_cards), device=DEV)
    beta[local[:, 0], local[:, 1]] = pair_beta
    beta[local[:, 1], local[:, 0]] = pair_beta
    torch.testing.assert_close(r["hand_log_ratio"][0], alpha[local[:, 0]] + alpha[local[:, 1]] + pair_beta,
                               atol=2e-5, rtol=2e-5)
    rec = torch.einsum("cr,r,dr->cd", r["beta_eigenvector"][0], r["beta_eigenvalue"][0], r["beta_eigenvector"][0])
    torch.testing.assert_close(rec, beta, atol=2e-5, rtol=2e-5)


def test_two_folders_match_exact_enumeration():
    from pbg_b200.folded import folded_statistics

    geometry, combo = _machine(3, 8.0, 4)
    local = (combo - geometry.first_card).long()
    first = torch.arange(1, geometry.private_hands + 1, dtype=torch.float32, device=DEV)
    second = torch.flip(first, dims=(0,))
    ranges = torch.zeros((1, 3, geometry.private_hands), device=DEV)
    ranges[0, 1], ranges[0, 2] = first, second
    status = torch.tensor([[0, 1, 1]], dtype=torch.int8, device=DEV)
    board = torch.full((1, 5), 255, dtype=torch.uint8, device=DEV)
    r = folded_statistics(geometry, board_cards=board, range_weights=ranges, status=status, combo_cards=combo,
                          beta_rank=geometry.deck_cards, line_dim=0)
    p = torch.stack((first / first.sum(), second / second.sum()))
    disjoint = local[:, None, :, None].ne(local[None, :, None, :]).all(-1).all(-1).float()
    base = torch.einsum("h,g,hg->", p[0], p[1], disjoint)
    for hand in range(0, geometry.private_hands, 17):
        survives = local.ne(local[hand][0]).all(-1) & local.ne(local[hand][1]).all(-1)
        part = torch.einsum("h,g,hg->", p[0] * survives, p[1] * survives, disjoint)
        torch.testing.assert_close(r["hand_log_ratio"][0, hand], torch.log(part / base), atol=3e-5, rtol=3e-5)


def test_three_loose_folders_calibrate_to_exact_enumeration():
    from pbg_b200.folded import folded_statistics

    geometry, combo = _machine(4, 8.0, 4)
    local = (combo - geometry.first_card).long()
    ordinal = torch.arange(geometry.private_hands, dtype=torch.float32, device=DEV)
    p = torch.stack([1.0 + 0.1 * torch.sin(ordinal * (f + 1) * 0.07) for f in range(3)])
    p /= p.sum(-1, keepdim=True)
    ranges = torch.zeros((1, 4, geometry.private_hands), device=DEV)
    ranges[0, 1:] = p
    status = torch.tensor([[0, 1, 1, 1]], dtype=torch.int8, device=DEV)
    board = torch.full((1, 5), 255, dtype=torch.uint8, device=DEV)
    r = folded_statistics(geometry, board_cards=board, range_weights=ranges, status=status, combo_cards=combo,
                          beta_rank=geometry.deck_cards, line_dim=0)
    disjoint = local[:, None, :, None].ne(local[None, :, None, :]).all(-1).all(-1).float()

    def exact(w):
        return torch.einsum("h,i,j,hi,hj,ij->", w[0], w[1], w[2], disjoint, disjoint, disjoint)

    base = exact(p)
    for hand in range(0, geometry.private_hands, 17):
        survives = local.ne(local[hand][0]).all(-1) & local.ne(local[hand][1]).all(-1)
        torch.testing.assert_close(r["hand_log_ratio"][0, hand], torch.log(exact(p * survives) / base),
                                   atol=1e-3, rtol=1e-3)


def test_tight_mask_on_a_live_seat_is_reported():
    # folded.py:266-269: the device check is recorded (no fault, every index in range) and raised on the host
    from pbg_b200.checks import input_errors, raise_input_errors
    from pbg_b200.folded import folded_statistics

    geometry, combo = _machine(3, 8.0, 4)
    input_errors(DEV)
    status = torch.tensor([[0, 0, 1]], dtype=torch.int8, device=DEV)
    tight = torch.tensor([[True, False, True]], device=DEV)
    folded_statistics(geometry, board_cards=torch.full((1, 5), 255, dtype=torch.uint8, device=DEV),
                      range_weights=torch.rand((1, 3, geometry.private_hands), device=DEV), status=status,
                      combo_cards=combo, beta_rank=4, line_dim=0, tight_mask=tight)
    with pytest.raises(ValueError, match="tight-folder mask includes a live seat"):
        raise_input_errors(DEV)


def test_timing_six_handed_full_deck():
    from pbg_b200.folded import folded_statistics, phi_queries

    geometry, combo = _machine(6, 100.0, 13)
    batch = 64
    g = torch.Generator(device=DEV).manual_seed(3)
    status = torch.zeros((batch, 6), dtype=torch.int8, device=DEV)
    status[:, 2:] = 1
    board = torch.full((batch, 5), 255, dtype=torch.uint8, device=DEV)
    board[:, :3] = torch.tensor([3, 17, 40], dtype=torch.uint8)
    weights = torch.rand((batch, 6, 1326), generator=g, device=DEV)
    prob, folder, valid = _probability(weights, status, board, 0, combo)
    base = 52 - valid.sum(-1, dtype=torch.float32)
    for _ in range(2):
        phi_queries(prob, folder, folder, base, 52)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    phi_queries(prob, folder, folder, base, 52)
    b.record()
    torch.cuda.synchronize()
    t = time.perf_counter()
    folded_statistics(geometry, board_cards=board, range_weights=weights, status=status, combo_cards=combo,
                      beta_rank=52, line_dim=0)
    torch.cuda.synchronize()
    print(f"\nfolded phi queries, 6-handed R13, 4 folders (all tight), {batch} rows x 1379 queries: "
          f"{a.elapsed_time(b):.3f} ms; whole folded_statistics {1e3 * (time.perf_counter() - t):.1f} ms")


@pytest.mark.parametrize("n,batch", [(52, 40), (16, 7), (20, 3), (33, 5)])
def test_symmetric_eigh_matches_torch(n, batch):
    from pbg_b200.folded import symmetric_eigh

    g = torch.Generator(device=DEV).manual_seed(n)
    a = torch.randn((batch, n, n), generator=g, device=DEV) * 0.1
    a = a + a.transpose(1, 2)
    a[0, :5] = 0.0          # zero rows and columns (board cards): a degenerate zero eigenvalue
    a[0, :, :5] = 0.0
    if batch > 1:
        a[1] = torch.diag(torch.tensor([1.0, 1.0, -2.0] + [0.5] * (n - 3), device=DEV))  # repeated eigenvalues
    values, vectors = symmetric_eigh(a)
    want = torch.linalg.eigh(a.double()).eigenvalues.float()
    scale = float(want.abs().max())
    torch.testing.assert_close(values, want, rtol=0, atol=2e-6 * scale * n)
    eye = torch.eye(n, device=DEV).expand(batch, -1, -1)
    # fp32 rotations accumulate about one rounding per sweep and index into V: orthogonal to 5e-5 at n = 52
    torch.testing.assert_close(vectors.transpose(1, 2) @ vectors, eye, rtol=0, atol=5e-5)
    torch.testing.assert_close(vectors @ torch.diag_embed(values) @ vectors.transpose(1, 2), a, rtol=0,
                               atol=2e-6 * scale * n)
