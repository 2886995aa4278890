"""CPU checks of the layered-target restatement and host-side argument handling.

The oracle is pinned by the expected values pbg's own executor tests assert
(tests/test_layered_targets.py in the reference); the seeded forests check
that the restatement is deterministic and free of failures on valid plans.
"""

import numpy as np
import pytest

import oracle
import target_forest as tf


@pytest.mark.parametrize("case", tf.known_answer_cases(), ids=lambda c: c[0])
def test_oracle_known_answers(case):
    _, plan, check = case
    failure, arenas = plan.run_oracle(oracle)
    check(failure, arenas)


@pytest.mark.parametrize("sampled", [True, False])
@pytest.mark.parametrize("branched", [False, True])
@pytest.mark.parametrize("reuse", [False, True])
def test_oracle_forest_valid_and_deterministic(sampled, branched, reuse):
    forest = tf.Forest(11, sampled=sampled, branched=branched, reuse=reuse, layers=5)
    f1, a1 = forest.run_oracle(oracle)
    f2, a2 = forest.run_oracle(oracle)
    assert (f1 == 2**31 - 1).all()
    assert np.array_equal(f1, f2)
    for name, group in a1.items():
        if group is None:
            continue
        for x, y in zip(group, a2[name]):
            if x is not None:
                np.testing.assert_array_equal(x, y)
    # every trained owner row received a sigma target
    written = sum(int(np.isfinite(s).all(-1).sum()) for s in a1["sigma_v"])
    owners = sum(1 for lane, inp, own in zip(forest.nodes[0], forest.nodes[4], forest.nodes[6]) if inp >= 0 and own >= 0)
    assert written == owners


def test_oracle_lambda_one_sampled_sigma_is_subtree_mean():
    # A chain of two single-child nodes returns the leaf value unchanged at lambda = 1.
    leaf = {(0, 0, 0): (np.array([[5.0]], np.float32), None, None, 0.0, 0.0)}
    a = dict(replica=0, owner=0, children=[(0, 0, 1, 1.0)], destination_row=1, sigma_target_row=0, action_begin=0)
    b = dict(replica=0, owner=0, children=[(1, 1, 1, 1.0)], destination_row=2, sigma_target_row=1, action_begin=1)
    plan = tf.HandPlan(width=1, p_train=1, sampled=True, branched=False, lam=1.0, layers=[[a], [b]], leaves=leaf,
                       head={(0, 0): (np.full(1, 9.0), 0.0, 0.0)})
    failure, arenas = plan.run_oracle(oracle)
    assert failure.tolist() == [2**31 - 1]
    assert arenas["sigma_v"][0][:, 0].tolist() == [5.0, 5.0]
    assert arenas["action_a"][0][:, 0].tolist() == [-4.0, -4.0]


def test_host_conversion_table_and_lambda_checks():
    from pbg_b200.targets import TargetError, _lambda, conversion_table

    table = conversion_table(tf.WIDTHS, {(1, 0): tf.CONVERT_1_TO_0})
    assert np.array_equal(table.numpy(), tf.conversion())
    with pytest.raises(TargetError):
        conversion_table(tf.WIDTHS, {(1, 0): (0, 1)})
    with pytest.raises(TargetError):
        conversion_table(tf.WIDTHS, {(1, 0): (0, 0, 1, 2, 3)})
    for bad in (-0.1, 1.5, float("nan")):
        with pytest.raises(TargetError):
            _lambda(bad)
    assert _lambda(0.25) == 0.25
