"""The reference's own training engine with this build's kernels swapped in (pbg_b200.engine).

The reference package (pbg, installed under baseline/_ref) runs one full
iteration -- rollout, completion, targets, learner, optimizer step -- twice
from the same seed in fresh processes (tests/engine_dropin_run.py), with the
sampled and with the Rao-Blackwell private estimator: once
unmodified and once after ``pbg_b200.engine.install()`` has routed its state
machine, composite policy and layered targets to libpbgb200.  The drop-in
must leave the engine's results where the reference puts them:

* the same rollout: equal player-node, leaf, layer and edge counts (cards,
  actions and chips are bit-exact by the parity tests; an action could only
  differ at a near-tie of the sampler, which these counts would expose);
* the same learner step: loss metrics within rtol 1e-4, and the flat
  gradient the AdamW transition receives within rtol 1e-3 plus 1e-5 of its
  largest entry.  The first AdamW step moves each parameter by +-lr times the
  sign of its gradient, so parameters are compared where the sign is decided:
  wherever the gradient exceeds 1e-3 of its largest entry they must agree to
  1e-6; elsewhere (gradients at rounding level, such as an attention key bias,
  whose gradient is zero by the softmax's shift invariance) they may differ
  by at most 2 lr.

Skipped when the reference package is not installed (its layered-targets
extension is compiled from pbg/core/csrc/layered_targets.cu at run time, so
the install must include the package's .cu files).
"""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref", "pbg")
# the reference JIT-compiles its layered-targets extension from the package's own CUDA source
REF_TARGETS_SOURCE = os.path.join(REF, "core", "csrc", "layered_targets.cu")


def _run(out, arm, estimator, geometry=(2, 8.0, 4), roots=16):
    env = dict(os.environ, TORCH_CUDA_ARCH_LIST=os.environ.get("TORCH_CUDA_ARCH_LIST", "10.0"))
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "engine_dropin_run.py"), out, arm, str(roots),
                           "1", "eager", estimator, *(str(g) for g in geometry)],
                          capture_output=True, text=True, timeout=900, env=env)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-6000:]
    return torch.load(os.path.join(out, f"{arm}.pt"), weights_only=False)


@pytest.mark.skipif(not os.path.isfile(REF_TARGETS_SOURCE),
                    reason="the reference package (with its CUDA sources) is not installed under baseline/_ref")
@pytest.mark.parametrize("arm,estimator,geometry,roots", [
    ("b200", "sampled", (2, 8.0, 4), 16), ("b200_learner", "sampled", (2, 8.0, 4), 16),
    ("b200", "rao_blackwell", (2, 8.0, 4), 16), ("b200_learner", "rao_blackwell", (2, 8.0, 4), 16),
    ("b200_learner", "rao_blackwell", (6, 100.0, 13), 8),  # cfg3's geometry: 6-max, 100 bb, 13 ranks
])
def test_reference_engine_runs_on_b200_kernels(tmp_path, arm, estimator, geometry, roots):
    """b200: state machine, policy and targets swapped; b200_learner: the loss program as well
    (``LearnerOperation.forward_loss`` -> one pbg_poker_learner_objective launch).  With the
    Rao-Blackwell estimator the leaves go through this build's ``rb_leaf`` and the reference's
    completion binding, whose evaluator (``complete``, this build's module in both runs) draws 64
    samples per leaf."""

    ref = _run(str(tmp_path), "reference", estimator, geometry, roots)
    b200 = _run(str(tmp_path), arm, estimator, geometry, roots)
    assert b200["installed"] and any("PokerStateMachine" in name for name in b200["installed"])
    assert ("forward_loss" in " ".join(b200["installed"])) == (arm == "b200_learner")
    assert (b200["fused_calls"] > 0) == (arm == "b200_learner")
    for key in ("player_nodes", "leaves", "target_layers", "executed_edges", "presentations"):
        assert [lane[key] for lane in b200["lanes"]] == [lane[key] for lane in ref["lanes"]], key
    for lane_b, lane_r in zip(b200["lanes"], ref["lanes"], strict=True):
        for loss_b, loss_r in zip(lane_b["losses"], lane_r["losses"], strict=True):
            for name, value in loss_r.items():
                # the log-ratio diagnostics sit at rounding level on a first minibatch (old and new log pi
                # agree to a few ulp of |log pi| ~ 5): an absolute 1e-5 there
                atol = 1e-5 if name in ("approximate_kl", "negative_advantage_log_ratio_max") else 1e-6
                assert abs(loss_b[name] - value) <= 1e-4 * abs(value) + atol, (name, loss_b[name], value)
    lr = 3.0e-4
    assert len(b200["gradients"]) == len(ref["gradients"]) >= 1
    for g_b, g_r in zip(b200["gradients"], ref["gradients"], strict=True):
        scale = float(g_r.abs().max())
        torch.testing.assert_close(g_b, g_r, rtol=1e-3, atol=1e-5 * scale)
    g_r = ref["gradients"][0][0]
    decided = g_r.abs() > 1e-3 * float(g_r.abs().max())
    assert sum(n for _, n in ref["layout"]) == g_r.numel()
    offset = 0
    for name, n in ref["layout"]:
        value = ref["state"][name]
        assert torch.equal(b200["state0"][name], ref["state0"][name]), f"initial {name} differs"
        sure = decided[offset:offset + n].reshape(value.shape)
        diff = (b200["state"][name] - value).abs()
        if bool(sure.any()):
            assert float(diff[sure].max()) <= 1e-6, name
        assert float(diff.max()) <= 2 * lr + 1e-6, name
        offset += n
    moved = max(float((ref["state"][n] - ref["state0"][n]).abs().max()) for n in ref["state"])
    assert moved > 1e-5  # the optimizer step did change the model
