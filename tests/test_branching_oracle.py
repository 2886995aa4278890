"""CPU checks of the alias-table and decision-log-mass restatements.

Pins: the reference's own alias test (tests/test_branched_sampled_modes.py:404-425:
the table reproduces softmax(log w) to 1e-15 even with a -1000 log weight)
and the closed form of the log mass on a hand-built tree.
"""

import math

import numpy as np

import oracle as O


def test_alias_table_preserves_softmax_mass():
    # the reference's own bound is for its 4-weight case; longer tables accumulate the
    # construction's float64 round-off in the last large entry (about 1e-14 at n = 4096)
    for log_w, atol in ((np.array([-1000.0, -3.0, -1.0, 0.0]), 1e-15), (np.linspace(-40, 0, 4096), 1e-12),
                        (np.random.default_rng(1).normal(0, 4, 10_000), 1e-12)):
        z = np.exp(log_w - np.logaddexp.reduce(log_w))
        prob, alias, _ = O.alias_table(z * log_w.size)
        observed = prob / log_w.size
        np.add.at(observed, alias, (1 - prob) / log_w.size)
        np.testing.assert_allclose(observed, z, atol=atol, rtol=1e-12)
        assert ((prob >= 0) & (prob <= 1)).all() and ((alias >= 0) & (alias < log_w.size)).all()


def test_alias_table_uniform_is_identity():
    prob, alias, _ = O.alias_table(np.ones(17))
    assert (prob == 1.0).all() and np.array_equal(alias, np.arange(17))


def test_decision_log_mass_closed_form():
    # root 0 (degree 3) -> 1 (degree 2) -> 3; root 0 -> 2; second root 4 -> 5
    parent = np.array([-1, 0, 0, 1, -1, 4], np.int32)
    degree = np.array([3, 2, 1, 1, 5, 1], np.int32)
    out, code = O.decision_log_mass(parent, degree)
    l3, l2, l5 = (np.float32(math.log(3)), np.float32(math.log(2)), np.float32(math.log(5)))
    assert code == 0
    assert out[0] == 0 and out[4] == 0
    assert out[1] == np.float32(0) - l3 and out[2] == np.float32(0) - l3
    assert out[3] == (np.float32(0) - l3) - l2 and out[5] == np.float32(0) - l5


def test_decision_log_mass_failures():
    assert O.decision_log_mass(np.array([-1, 1], np.int32), np.array([1, 1], np.int32))[1] == 1
    assert O.decision_log_mass(np.array([-1, 0], np.int32), np.array([0, 1], np.int32))[1] == 2
