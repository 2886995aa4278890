"""Collision-conditioned posterior sampler (rb_sampling.py:86-223) on the GPU.

Against the reference's own outputs (golden, run on CPU) and the C restatement
on larger seeded cases: profiles, attempt counts, exhaustion flags and the
minimum failing address must be identical.  Both sides build the CDF with
double accumulation rounded to fp32 per entry.
"""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _run(geometry, inputs, max_attempts):
    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rb_sampling import CollisionConditionedProfileSampler

    sampler = CollisionConditionedProfileSampler(NLHEGeometry(*geometry), max_attempts=max_attempts)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(DEV) for k, v in inputs.items() if k not in ("seed", "iteration")}
    result = sampler.sample_children(range_weights=t["weights"], board_cards=t["board"], inherited_profile=t["inherited"],
                                     source=t["source"], ordinal=t["ordinal"], active=t["active"].bool(),
                                     root=t["root"], path=t["path"], seed=int(inputs["seed"]),
                                     iteration=int(inputs["iteration"]), retry_epoch=t["epoch"])
    obs = sampler.last_observation
    return (result.cpu().numpy(), obs.attempt_count.cpu().numpy(), obs.exhausted.cpu().numpy(),
            int(obs.minimum_failing_address.item()))


def test_posterior_matches_reference_golden(gold):
    d = gold("posterior")
    for c in range(int(d["cases"])):
        p = f"c{c}_"
        geo, si = d[p + "geometry"], d[p + "seed_iteration"]
        inputs = {k: d[p + k] for k in ("weights", "board", "inherited", "source", "ordinal", "active", "root",
                                         "path", "epoch")}
        inputs.update(seed=si[0], iteration=si[1])
        out, count, exh, worst = _run((int(geo[0]), float(geo[1]), int(geo[2])), inputs, int(d[p + "max_attempts"]))
        assert np.array_equal(out, d[p + "result"]), c
        assert np.array_equal(count, d[p + "attempt_count"]), c
        assert np.array_equal(exh, d[p + "exhausted"]), c
        assert worst == int(d[p + "minimum_failing"]), c


def _seeded(geometry, parents, rows, seed, sparse=0.5):
    from pbg_b200.poker import NLHEGeometry

    geo = NLHEGeometry(*geometry)
    rng = np.random.default_rng(seed)
    H, D, first = geo.private_hands, geo.deck_cards, geo.first_card
    w = rng.random((parents, geo.players, H), dtype=np.float32)
    w[rng.random(w.shape) < sparse] = 0.0
    w[..., ::7] += 0.01  # board-legal mass survives any board
    board = np.full((parents, 5), 255, np.uint8)
    for b in range(parents):
        shown = [0, 3, 4, 5][b % 4]
        board[b, :shown] = rng.permutation(D)[:shown] + first
    return {"weights": w, "board": board,
            "inherited": rng.integers(0, H, (parents, geo.players), dtype=np.int32),
            "source": rng.integers(0, parents, rows, dtype=np.int64),
            "ordinal": rng.integers(0, 4, rows, dtype=np.int64),
            "active": (rng.random(rows) < 0.9).astype(np.uint8),
            "root": rng.integers(0, 2**62, rows, dtype=np.int64),
            "path": rng.integers(-2**62, 2**62, rows, dtype=np.int64),
            "epoch": rng.integers(0, 3, rows, dtype=np.int64), "seed": 11 + seed, "iteration": 3}


@pytest.mark.parametrize("geometry,attempts", [((6, 100.0, 13), 256), ((2, 100.0, 13), 256), ((3, 20.0, 6), 4),
                                               ((5, 50.0, 9), 256)])
def test_posterior_matches_oracle_on_seeded_forests(geometry, attempts):
    inputs = _seeded(geometry, parents=40, rows=3000, seed=geometry[0] * 10 + attempts)
    out, count, exh, worst = _run(geometry, inputs, attempts)
    ref = O.posterior_sample(geometry, inputs["weights"], inputs["board"], inputs["inherited"], inputs["source"],
                             inputs["ordinal"], inputs["active"], inputs["root"], inputs["path"], inputs["seed"],
                             inputs["iteration"], inputs["epoch"], attempts)
    assert np.array_equal(out, ref[0])
    assert np.array_equal(count, ref[1])
    assert np.array_equal(exh, ref[2])
    assert worst == ref[3]
    if attempts == 256 and geometry[0] >= 5:
        assert count.max() > 1  # collisions happened and were rejected


def test_posterior_rows_are_independent_of_batching():
    geometry = (6, 100.0, 13)
    inputs = _seeded(geometry, parents=16, rows=500, seed=5)
    full = _run(geometry, inputs, 256)
    pick = np.arange(0, 500, 7)
    sub = dict(inputs)
    for k in ("source", "ordinal", "active", "root", "path", "epoch"):
        sub[k] = inputs[k][pick]
    part = _run(geometry, sub, 256)
    assert np.array_equal(part[0], full[0][pick])
    assert np.array_equal(part[1], full[1][pick])


def test_posterior_without_board_legal_mass_raises():
    from pbg_b200.rb_sampling import PosteriorSamplingError

    geometry = (2, 100.0, 13)
    inputs = _seeded(geometry, parents=2, rows=8, seed=9)
    inputs["weights"][1, 0, :] = 0.0
    inputs["source"][:] = 1
    inputs["active"][:] = 1
    inputs["ordinal"][:] = 1
    with pytest.raises(PosteriorSamplingError):
        _run(geometry, inputs, 256)
