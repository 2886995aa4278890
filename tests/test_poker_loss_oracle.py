"""The float64 poker-learner oracle against the reference's own loss program (no GPU).

tests/golden/poker_loss.npz holds ``LearnerOperation.forward_loss`` results and
autograd gradients of ``(total * lane_weight).sum()`` computed by the
reference on CPU (tests/golden/make_golden.py ``gen_poker_loss``), for sampled
and Rao-Blackwell rows, sequential and branched batches, one and two lanes,
and ``PokerPolicyOperator.learner`` gradients.  The oracle must reproduce them
within the reference's own policy-gradient tolerance (atol 2e-6, rtol 2e-5;
tests/test_sequential_sampled_training.py:353-363 of the reference), widened
only by fp32 rounding of the terms a gradient is summed from (64 ulp of their
magnitude, ``poker_loss_oracle.within_rounding``): the reference computes in
fp32 and some mixture gradients are small differences of large terms.
"""

import numpy as np
import pytest

import poker_loss_oracle as P

from conftest import golden

GOLD = golden("poker_loss")
CASES = [str(c) for c in GOLD["cases"]]


@pytest.mark.parametrize("case", CASES)
def test_oracle_reproduces_reference_loss_and_gradients(case):
    batch = P.from_golden(GOLD, case)
    result, grads, mags = P.poker_learner_objective(batch, magnitude=True)
    np.testing.assert_allclose(result, GOLD[f"pl_{case}_result"], rtol=2e-5, atol=2e-6)
    for name in ("value", "trace_pred", "cost_pred"):
        if name in grads:
            np.testing.assert_allclose(grads[name], GOLD[f"pl_{case}_grad_{name}"], rtol=2e-5, atol=2e-6,
                                       err_msg=f"{case}:{name}")
    for name in P.FIELDS:
        ok = P.within_rounding(grads[name], GOLD[f"pl_{case}_grad_{name}"], mags[name], k=16)
        assert ok.all(), f"{case}:{name}: {np.argwhere(~ok)[:4].tolist()}"


@pytest.mark.parametrize("case", ["pl202", "pl18"])
def test_oracle_policy_learner_matches_reference_autograd(case):
    pre = f"plr_{case}_"
    raw = {k: GOLD[pre + k] for k in P.FIELDS}
    ref = {k: GOLD[pre + "ref_" + k] for k in P.FIELDS}
    w_sel, w_ent, w_kl = GOLD[pre + "weights"].astype(np.float64)
    (sel, ent, kl), grads, mags = P.policy_learner_vjp(raw, ref, GOLD[pre + "mask"].astype(bool), GOLD[pre + "action"],
                                                       w_sel, w_ent, w_kl, magnitude=True)
    np.testing.assert_allclose(sel, GOLD[pre + "selected"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ent, GOLD[pre + "entropy"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(kl, GOLD[pre + "kl"], rtol=1e-5, atol=1e-6)
    for name in P.FIELDS:
        ok = P.within_rounding(grads[name], GOLD[pre + "grad_" + name], mags[name], k=16)
        assert ok.all(), f"{case}:{name}: {np.argwhere(~ok)[:4].tolist()}"


def test_rounding_allowance_only_widens_the_cancelling_fields():
    """The allowance is negligible for the logits and the all-in weight, where nothing cancels."""

    batch = P.from_golden(GOLD, "s202")
    _, grads, mags = P.poker_learner_objective(batch, magnitude=True)
    for name in ("type_logits", "iota"):
        allowance = 16 * 2.0 ** -24 * mags[name]
        assert (allowance <= 1e-5 * np.abs(grads[name]) + 1e-9).all(), name


def test_uniform_fallback_row_is_exercised():
    """Row 2 of the E=10 case has no fp32 mixture mass on its legal ticks: the uniform law."""

    batch = P.from_golden(GOLD, "s10")
    _, cache = P.policy_forward(batch.raw, batch.mask)
    assert cache.parts["mass"][2, 0] == 0.0
    assert np.allclose(cache.parts["cond"][2, 0][batch.mask[2, 2:]], 0.5)
