"""Layered-target kernel (one cooperative launch) against the CPU restatement.

Bit-exact: both sides evaluate the reference's fp32 operation order with no
contraction (the kernel is built with -fmad=false, as the reference's layer
operator is, pbg/core/cuda_layer.py:22).
"""

import numpy as np
import pytest
import torch

import oracle
import target_forest as tf

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _assert_same(a_ref: dict, a_dev: dict):
    for name, group in a_ref.items():
        if group is None:
            continue
        for i, (x, y) in enumerate(zip(group, a_dev[name])):
            if x is not None:
                np.testing.assert_array_equal(x, y, err_msg=f"{name}[{i}]")


@pytest.mark.parametrize("case", tf.known_answer_cases(), ids=lambda c: c[0])
def test_known_answers_on_device(case):
    _, plan, check = case
    failure, arenas = plan.run_device(DEV)
    check(failure, arenas)
    ref_failure, ref = plan.run_oracle(oracle)
    assert np.array_equal(failure, ref_failure)
    if (failure == 2**31 - 1).all():
        _assert_same(ref, arenas)


@pytest.mark.parametrize("sampled", [True, False])
@pytest.mark.parametrize("branched", [False, True])
@pytest.mark.parametrize("reuse", [False, True])
@pytest.mark.parametrize("seed", [0, 1])
def test_forest_matches_oracle_bit_exact(sampled, branched, reuse, seed):
    forest = tf.Forest(100 + seed, n_replica=4, sampled=sampled, branched=branched, reuse=reuse, layers=6,
                       width_per_layer=24)
    ref_failure, ref = forest.run_oracle(oracle)
    failure, arenas = forest.run_device(DEV)
    assert np.array_equal(failure, ref_failure)
    _assert_same(ref, arenas)


def test_wide_forest_grid_strided():
    # more nodes per layer than the grid has warps: every warp loops over nodes
    forest = tf.Forest(7, n_replica=48, sampled=False, branched=True, layers=5, width_per_layer=400)
    assert forest.layer_ptr[1] > 148 * 4 * 8
    ref_failure, ref = forest.run_oracle(oracle)
    failure, arenas = forest.run_device(DEV)
    assert np.array_equal(failure, ref_failure)
    _assert_same(ref, arenas)


def test_failure_lane_isolated_in_forest():
    forest = tf.Forest(5, n_replica=4, sampled=True, branched=False, layers=4)
    arenas = forest.copy_arenas()
    lane, t, row, arena = next(x for x in forest.leaves if x[0] == 2)
    arenas["work0"][t][lane, row, arena] = np.nan
    ref_failure, ref = forest.run_oracle(oracle, {k: None if v is None else [None if a is None else a.copy() for a in v]
                                                  for k, v in arenas.items()})
    failure, dev = forest.run_device(DEV, arenas)
    assert ref_failure[2] != 2**31 - 1
    assert np.array_equal(failure, ref_failure)
    for name in ("work0",):
        for x, y in zip(ref[name], dev[name]):
            keep = [0, 1, 3]
            np.testing.assert_array_equal(x[keep], y[keep])
    for i in (0, 1, 3):
        for part in range(forest.input_count):
            k = i * forest.input_count + part
            np.testing.assert_array_equal(ref["sigma_v"][k], dev["sigma_v"][k])


def test_bound_relaunch_leaves_barrier_clean():
    from pbg_b200.targets import LayeredTargets

    forest = tf.Forest(9, n_replica=3, sampled=False, branched=True, layers=6, reuse=True)
    _, ref = forest.run_oracle(oracle)
    arenas = forest.copy_arenas()
    n_in, n_out = forest.input_count, forest.output_count
    empty = torch.empty(0, dtype=torch.float32, device=DEV)

    def dev(group, count):
        return [empty] * count if group is None else [empty if a is None else torch.from_numpy(a).to(DEV)
                                                      for a in group]

    counts = dict(work0=n_out, work1=n_out, trace=n_out, cost=n_out, delta=n_out, head_v=n_in, head_t=n_in,
                  head_c=n_in, sigma_v=3 * n_in, sigma_t=3 * n_in, sigma_c=3 * n_in,
                  action_p=3 * forest.action_partitions, action_a=3 * forest.action_partitions)
    pristine = {k: dev(arenas[k], c) for k, c in counts.items()}
    live = {k: [t.clone() for t in v] for k, v in pristine.items()}
    bound = LayeredTargets(torch.from_numpy(forest.layer_ptr), [torch.from_numpy(a).to(DEV) for a in forest.nodes],
                           [torch.from_numpy(a).to(DEV) for a in forest.children],
                           *[live[k] for k in counts], torch.from_numpy(forest.conversion), forest.work_cap,
                           forest.head_cap, forest.width, 3, n_in, n_out, forest.action_partitions, forest.p_train,
                           max(forest.width), forest.lam, forest.sampled, forest.branched)
    for _ in range(3):
        for k in counts:
            for dst, src in zip(live[k], pristine[k]):
                dst.copy_(src)
        failure = bound.launch()
        torch.cuda.synchronize()
        assert (failure.cpu() == 2**31 - 1).all()
        ws = bound.workspace.cpu()
        assert int(ws[0]) == 0 and int(ws[64]) == 0 and int(ws[65]) == 0 and not ws[96:].any()
        for k in counts:
            if ref[k] is None:
                continue
            for x, t in zip(ref[k], live[k]):
                if x is not None:
                    np.testing.assert_array_equal(x, t.cpu().numpy(), err_msg=k)


def test_lambda_out_of_range_raises_before_launch():
    from pbg_b200.targets import TargetError

    forest = tf.Forest(1)
    forest.lam = 1.5
    with pytest.raises(TargetError):
        forest.run_device(DEV)


@pytest.mark.parametrize("sampled,branched", [(False, True), (True, False), (False, False), (True, True)])
def test_synthetic_tree_plan_matches_oracle(sampled, branched):
    # the bench workload's generator, at a small size, checked against the restatement
    from pbg_b200.targets import run_layers, synthetic_tree_plan

    args, info = synthetic_tree_plan(6, 5, 3, 2, 4, device=DEV, sampled=sampled, branched=branched, seed=1)
    groups = {name: [None if t.numel() == 0 else t.cpu().numpy().copy() for t in group]
              for name, group in zip(oracle.TARGET_GROUPS, args[3:16])}
    for name in groups:
        if all(a is None for a in groups[name]):
            groups[name] = None
    ref_failure = oracle.layered_targets(
        args[0].numpy(), [t.cpu().numpy() for t in args[1]], [t.cpu().numpy() for t in args[2]], groups,
        args[16].cpu().numpy(), args[17], args[18], args[19], n_replica=args[20], input_count=args[21],
        output_count=args[22], action_partitions=args[23], p_train=args[24], lam=args[26], sampled=args[27],
        branched=args[28])
    failure = run_layers(*args)
    torch.cuda.synchronize()
    assert (ref_failure == 2**31 - 1).all()
    assert np.array_equal(failure.cpu().numpy(), ref_failure)
    for name, group in zip(oracle.TARGET_GROUPS, args[3:16]):
        if groups[name] is None:
            continue
        for i, (x, t) in enumerate(zip(groups[name], group)):
            if x is not None:
                np.testing.assert_array_equal(x, t.cpu().numpy(), err_msg=f"{name}[{i}]")


def test_run_layers_rebinds_nothing_and_reads_live_arenas():
    # repeated calls over the same arenas reuse one binding; the kernel reads the arenas' current contents
    from pbg_b200 import targets as T

    forest = tf.Forest(23, n_replica=3, sampled=False, branched=True, layers=4)
    args, groups, arenas = forest.device_args(DEV)
    T.clear_bindings()
    first = T.run_layers(*args)
    assert len(T._BINDINGS) == 1
    lane, t, row, arena = forest.leaves[0]
    scale = 2.0
    groups["work1"][t][lane, row, arena] *= scale
    second = T.run_layers(*args)
    torch.cuda.synchronize()
    assert len(T._BINDINGS) == 1
    assert first.data_ptr() != second.data_ptr()
    host = forest.copy_arenas()
    host["work1"][t][lane, row, arena] *= np.float32(scale)
    ref_failure, ref = forest.run_oracle(oracle, host)
    assert np.array_equal(second.cpu().numpy(), ref_failure)
    for name, group in groups.items():
        if ref[name] is None:
            continue
        for x, y in zip(ref[name], group):
            if x is not None:
                np.testing.assert_array_equal(x, y.cpu().numpy(), err_msg=name)


def test_failure_codes_are_cleared_for_the_next_launch():
    from pbg_b200.targets import INT32_MAX, LayeredTargets

    forest = tf.Forest(31, n_replica=3, sampled=True, branched=False, layers=3)
    args, groups, _ = forest.device_args(DEV)
    bound = LayeredTargets(*args)
    lane, t, row, arena = forest.leaves[0]
    good = groups["work0"][t][lane, row, arena].clone()
    groups["work0"][t][lane, row, arena] = float("nan")
    first = bound.launch().cpu().clone()
    assert first[lane] != INT32_MAX and (first[[i for i in range(3) if i != lane]] == INT32_MAX).all()
    groups["work0"][t][lane, row, arena] = good
    second = bound.launch().cpu()
    assert (second == INT32_MAX).all()
    ws = bound.workspace.cpu()  # counters and failure codes clean; the barrier generation keeps counting
    assert int(ws[0]) == 0 and int(ws[64]) == 0 and int(ws[65]) == 0 and not ws[96:].any()
