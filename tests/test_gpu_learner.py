"""The fused poker learner objective on the GPU against the reference and the float64 oracle.

* Against the reference: tests/golden/poker_loss.npz holds the reference's own
  ``LearnerOperation.forward_loss`` results and autograd gradients (sampled and
  Rao-Blackwell rows, sequential and branched batches with trace/cost heads,
  one and two lanes, clipped and MSE value, log cap, reference KL, the uniform
  fallback row) and ``PokerPolicyOperator.learner`` gradients.  Loss values:
  rtol 2e-5 / atol 2e-6; value and head gradients: the same; raw-field
  gradients: the same plus 16 ulp of the magnitude of the terms each is
  summed from (``poker_loss_oracle.within_rounding``), because the reference's
  fp32 autograd forms the mixture location/scale gradients from nearly
  cancelling product-rule terms.
* Against the float64 restatement on larger seeded batches (E = 202 and 102
  sampled, Rao-Blackwell with H = 120 and 1326 columns, branched spans, four
  lanes): the kernel forms the cancellation-free telescoped derivative, so it
  is held to atol 2e-6 / rtol 2e-5 plus 2 ulp of the term magnitude.
* The autograd wrappers: ``poker_learner_loss(...).total`` backpropagates the
  same gradients, scaled per lane by the upstream gradient, and
  ``PokerPolicyOperator.learner`` is differentiable.
"""

import numpy as np
import pytest
import torch

import poker_loss_oracle as P

from conftest import golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLD = golden("poker_loss")
CASES = [str(c) for c in GOLD["cases"]]


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def _run(batch: P.LearnerBatch):
    from pbg_b200.learner import PokerLearnerObjective

    obj = PokerLearnerObjective(DEV)
    W = batch.raw["type_logits"].shape[1]
    raw = {k: _t(v) for k, v in batch.raw.items()}
    ref = None if batch.ref_raw is None else {k: _t(v) for k, v in batch.ref_raw.items()}
    S = batch.mask.shape[0]
    A = batch.action.shape[0]
    kw = {}
    if batch.trace_pred is not None:
        kw = dict(trace_pred=_t(batch.trace_pred), cost_pred=_t(batch.cost_pred), trace_target=_t(batch.trace_target),
                  cost_target=_t(batch.cost_target))
    unit = np.array_equal(batch.action_ptr, np.arange(S + 1))
    res, grads = obj(raw, _t(batch.mask.astype(bool)), _t(batch.action), _t(batch.old), _t(batch.adv),
                     _t(batch.value), _t(batch.old_value), _t(batch.target), _t(batch.controls),
                     _t(batch.lane_weight), posterior=_t(batch.post) if W > 1 else None,
                     action_ptr=None if unit and A == S and batch.trace_pred is None else _t(batch.action_ptr),
                     reference_raw=ref, **kw)
    torch.cuda.synchronize()
    result = np.stack([getattr(res, f).cpu().numpy() for f in P.RESULT], 1)
    return result, {k: v.cpu().numpy() for k, v in grads.items()}


@pytest.mark.parametrize("case", CASES)
def test_kernel_matches_reference_loss_and_gradients(case):
    batch = P.from_golden(GOLD, case)
    result, grads = _run(batch)
    np.testing.assert_allclose(result, GOLD[f"pl_{case}_result"], rtol=2e-5, atol=2e-6)
    _, _, mags = P.poker_learner_objective(batch, magnitude=True)
    for name in ("value", "trace_pred", "cost_pred"):
        if name in grads:
            np.testing.assert_allclose(grads[name], GOLD[f"pl_{case}_grad_{name}"], rtol=2e-5, atol=2e-6,
                                       err_msg=f"{case}:{name}")
    for name in P.FIELDS:
        ok = P.within_rounding(grads[name], GOLD[f"pl_{case}_grad_{name}"], mags[name], k=16)
        assert ok.all(), f"{case}:{name} at {np.argwhere(~ok)[:4].tolist()}"


def _masks(gi, E):
    from conftest import golden as gold_file

    packed = gold_file("poker")[f"g{gi}_masks"]
    masks = np.unpackbits(packed, axis=-1)[..., :E].astype(bool).reshape(-1, E)
    return masks[masks.any(1)]


ORACLE_CASES = [
    # (seed, S, W, E, M, lanes, max_span, reference, heads, mask geometry)
    (1, 512, 1, 202, 2, 2, 1, True, False, 3),
    (2, 256, 1, 102, 3, 4, 3, True, True, 5),
    (3, 24, 120, 18, 2, 2, 1, True, False, 0),
    (4, 8, 1326, 202, 2, 1, 2, False, True, 3),
]


@pytest.mark.parametrize("case", ORACLE_CASES, ids=lambda c: f"S{c[1]}W{c[2]}E{c[3]}L{c[5]}")
def test_kernel_matches_float64_restatement(case):
    seed, S, W, E, M, lanes, span, ref, heads, gi = case
    batch = P.seeded_batch(seed, S=S, W=W, E=E, M=M, lanes=lanes, max_span=span, reference=ref, heads=heads,
                           masks=_masks(gi, E))
    result, grads = _run(batch)
    want, wgrads, mags = P.poker_learner_objective(batch, magnitude=True)
    np.testing.assert_allclose(result, want, rtol=2e-5, atol=2e-6)
    for name in ("value", "trace_pred", "cost_pred"):
        if name in wgrads:
            np.testing.assert_allclose(grads[name], wgrads[name], rtol=2e-5, atol=2e-6, err_msg=name)
    for name in P.FIELDS:
        ok = P.within_rounding(grads[name], wgrads[name], mags[name], k=2)
        assert ok.all(), f"{name} at {np.argwhere(~ok)[:4].tolist()}"


def test_repeated_launches_are_deterministic():
    batch = P.seeded_batch(7, S=256, W=1, E=202, lanes=2, masks=_masks(3, 202))
    r1, g1 = _run(batch)
    r2, g2 = _run(batch)
    assert np.array_equal(r1, r2)
    for k in g1:
        assert np.array_equal(g1[k], g2[k]), k


def test_autograd_wrapper_scales_lanes_by_upstream_gradient():
    from pbg_b200.learner import PokerLearnerObjective, poker_learner_loss

    batch = P.from_golden(GOLD, "s202")
    raw = {k: _t(v).requires_grad_() for k, v in batch.raw.items()}
    value = _t(batch.value).requires_grad_()
    ref = {k: _t(v) for k, v in batch.ref_raw.items()}
    res = poker_learner_loss(PokerLearnerObjective(DEV), raw, value, mask=_t(batch.mask.astype(bool)),
                             action=_t(batch.action), old_log_policy=_t(batch.old), advantage_target=_t(batch.adv),
                             old_value=_t(batch.old_value), value_target=_t(batch.target),
                             controls=_t(batch.controls), reference_raw=ref)
    (res.total * _t(batch.lane_weight)).sum().backward()
    np.testing.assert_allclose(res.total.detach().cpu().numpy(), GOLD["pl_s202_result"][:, 0], rtol=2e-5, atol=2e-6)
    _, wgrads, mags = P.poker_learner_objective(batch, magnitude=True)
    for name in P.FIELDS:
        assert P.within_rounding(raw[name].grad.cpu().numpy(), wgrads[name], mags[name], k=2).all(), name
    np.testing.assert_allclose(value.grad.cpu().numpy(), wgrads["value"], rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("case", ["pl202", "pl18"])
def test_policy_learner_is_differentiable_and_matches_reference(case):
    from pbg_b200.poker import PokerLegality
    from pbg_b200.policy import PokerPolicyOperator

    pre = f"plr_{case}_"
    raw = {k: _t(GOLD[pre + k]).requires_grad_() for k in P.FIELDS}
    ref = {k: _t(GOLD[pre + "ref_" + k]) for k in P.FIELDS}
    mask = _t(GOLD[pre + "mask"]).bool()
    B, E = mask.shape
    legality = PokerLegality(torch.arange(E, dtype=torch.int32, device=DEV)[None].expand(B, -1).contiguous(), mask)
    ev = PokerPolicyOperator().learner(raw, legality, _t(GOLD[pre + "action"]), None, None, ref)
    np.testing.assert_allclose(ev.selected_log_policy.detach().cpu().numpy(), GOLD[pre + "selected"], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(ev.entropy.detach().cpu().numpy(), GOLD[pre + "entropy"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ev.reference_kl.detach().cpu().numpy(), GOLD[pre + "kl"], rtol=1e-5, atol=1e-6)
    w = _t(GOLD[pre + "weights"])
    (ev.selected_log_policy * w[0] + ev.entropy * w[1] + ev.reference_kl * w[2]).sum().backward()
    _, _, mags = P.policy_learner_vjp({k: GOLD[pre + k] for k in P.FIELDS}, {k: GOLD[pre + "ref_" + k] for k in P.FIELDS},
                                      GOLD[pre + "mask"].astype(bool), GOLD[pre + "action"], *GOLD[pre + "weights"],
                                      magnitude=True)
    for name in P.FIELDS:
        ok = P.within_rounding(raw[name].grad.cpu().numpy(), GOLD[pre + "grad_" + name], mags[name], k=16)
        assert ok.all(), f"{case}:{name} at {np.argwhere(~ok)[:4].tolist()}"


def test_bad_arguments_are_refused():
    from pbg_b200._native import NativeError
    from pbg_b200.learner import LearnerError

    batch = P.seeded_batch(9, S=6, W=1, E=18, lanes=1, masks=_masks(0, 18))
    batch.controls = np.repeat(batch.controls, 4, 0)  # 4 lanes do not divide 6 sigma rows
    batch.lane_weight = np.ones(4, np.float32)
    with pytest.raises((NativeError, LearnerError)):
        _run(batch)
