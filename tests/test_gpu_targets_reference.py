"""The layered-target kernel against the reference's own layer operator.

oracle/build_ref.py compiles pbg/core/csrc/layered_targets.cu (the
reference's kernel and its per-layer host loop) into oracle/_ref; these
tests skip when that module was not built.  Results must be bit-identical:
both kernels follow the same fp32 operation order with --fmad=false.
The timing test reports the single cooperative launch beside the
reference's one-launch-per-layer loop on the same forest.
"""

import time

import numpy as np
import pytest
import torch

import build_ref
import target_forest as tf

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
REF = build_ref.load()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref reference operator not built")


def _same(a: dict, b: dict):
    for name, group in a.items():
        if group is None:
            continue
        for i, (x, y) in enumerate(zip(group, b[name])):
            if x is not None:
                np.testing.assert_array_equal(x, y, err_msg=f"{name}[{i}]")


@needs_ref
@pytest.mark.parametrize("case", tf.known_answer_cases(), ids=lambda c: c[0])
def test_known_answers_match_reference_kernel(case):
    _, plan, check = case
    ref_failure, ref = plan.run_device(DEV, runner=REF.run_layers)
    check(ref_failure, ref)  # the expected values hold for the reference kernel itself
    failure, ours = plan.run_device(DEV)
    assert np.array_equal(failure, ref_failure)
    if (failure == 2**31 - 1).all():
        _same(ref, ours)


@needs_ref
@pytest.mark.parametrize("sampled", [True, False])
@pytest.mark.parametrize("branched", [False, True])
@pytest.mark.parametrize("reuse", [False, True])
def test_forest_matches_reference_kernel(sampled, branched, reuse):
    forest = tf.Forest(300, n_replica=6, sampled=sampled, branched=branched, reuse=reuse, layers=6,
                       width_per_layer=40)
    ref_failure, ref = forest.run_device(DEV, runner=REF.run_layers)
    failure, ours = forest.run_device(DEV)
    assert np.array_equal(failure, ref_failure)
    _same(ref, ours)


def _time(fn, reps=20, warmup=3):
    """(device us, wall us) per call.  Device: each call queued behind a device-side sleep, so the
    events bracket the GPU work of the call (its launches, and its host gaps only where the host
    falls behind the GPU); wall: back-to-back calls, host clock."""

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    device = []
    for _ in range(reps):
        torch.cuda._sleep(2_000_000)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        stop.record()
        torch.cuda.synchronize()
        device.append(start.elapsed_time(stop) * 1e3)
    wall = time.perf_counter()
    for _ in range(reps):
        fn()
    torch.cuda.synchronize()
    return sorted(device)[reps // 2], (time.perf_counter() - wall) / reps * 1e6


@needs_ref
def test_timing_single_launch_vs_reference_layer_loop():
    from pbg_b200.targets import LayeredTargets, clear_bindings, run_layers

    forest = tf.Forest(17, n_replica=64, sampled=False, branched=True, reuse=True, layers=8, width_per_layer=160,
                       extra_edges=False)
    args, _, _ = forest.device_args(DEV)
    nodes = int(forest.layer_ptr[-1])
    ref_us, ref_wall = _time(lambda: REF.run_layers(*args))
    ours_us, ours_wall = _time(lambda: run_layers(*args))

    def fresh():
        clear_bindings()  # a new plan every call: the binding is rebuilt each time
        run_layers(*args)

    fresh_us, fresh_wall = _time(fresh)
    bound = LayeredTargets(*args)
    bound_us, bound_wall = _time(lambda: bound.launch())
    print(f"\nlayered targets: {nodes} nodes, {forest.layer_ptr.size - 1} layers, 64 lanes, RB branched, P=2")
    print(f"  reference run_layers   : {ref_us:9.1f} us device  {ref_wall:9.1f} us wall")
    print(f"  pbg_b200 run_layers    : {ours_us:9.1f} us device  {ours_wall:9.1f} us wall  (binding reused)")
    print(f"  pbg_b200 run_layers    : {fresh_us:9.1f} us device  {fresh_wall:9.1f} us wall  (binding rebuilt)")
    print(f"  pbg_b200 bound launch  : {bound_us:9.1f} us device  {bound_wall:9.1f} us wall")
    assert bound_us < ref_us
