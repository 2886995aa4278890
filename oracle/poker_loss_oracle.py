"""Float64 restatement of the poker learner objective and its gradient (test infrastructure only).

This file is an oracle: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs import it, to check the CUDA library.

The objective is the reference's loss program for one physical batch:

* the composite policy of pbg/games/poker/queued/policy.py:113-204
  (``_discretized_logistic`` raise mixture, all-in atom, masked softmax over
  fold / check-call / raise ticks), its selected log-probability, entropy and
  reference KL (policy.py:206-244, clamped at epsilon 1e-12);
* ``LearnerOperation.forward_loss`` (pbg/core/learner.py:1824-2159): PPO
  clipped ratio with the negative-advantage log cap, posterior-weighted rows
  (Rao-Blackwell) or unit posterior (sampled), sigma means over ragged action
  spans, the MSE or clipped value objective under the sigma posterior,
  entropy and reference-KL bonuses, trace and cost heads of branched batches,
  and lane means;
* the backward of ``(total * lane_weight).sum()`` (pbg/core/training.py:403:
  objective weight times loss scale per lane).

The gradient is derived by hand in float64 and follows autograd's conventions
for the non-smooth points: ``clamp`` / ``clamp_min`` pass the gradient where
the input lies inside the closed interval; ``torch.minimum`` / ``maximum``
split a tie evenly; ``torch.where`` routes the gradient to the selected
branch only; ``masked_fill`` blocks it.

The reference computes in fp32, where a logistic tail below the smallest
subnormal (2^-149) is exactly zero; a raise law whose legal ticks all
underflow takes the uniform branch (policy.py:160-166).  The restatement
flushes the same tails to zero so that it takes the same branch.

``policy_backward(..., magnitude=True)`` runs the same chain on absolute
values (every difference becomes a sum): the result bounds the size of the
terms each gradient is summed from, so ``k * 2^-24 * magnitude`` bounds the
fp32 rounding error of an implementation that forms those terms, the
reference's autograd included.  Tests use it to tell rounding from error
where the gradient is a small difference of large terms.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

EPS = 1.0e-12
TINY = float(np.finfo(np.float32).tiny)
SUBNORMAL = 2.0 ** -149
FIELDS = ("type_logits", "omega", "mu", "s", "iota")
RESULT = ("total", "policy", "value", "entropy", "reference_kl", "approximate_kl", "clip_fraction",
          "negative_advantage_cap_fraction", "negative_advantage_log_ratio_max",
          "negative_advantage_influence_max")


def _sig(x):
    out = np.empty_like(x)
    pos = x >= 0
    out[pos] = 1.0 / (1.0 + np.exp(-x[pos]))
    e = np.exp(x[~pos])
    out[~pos] = e / (1.0 + e)
    return np.where(out < SUBNORMAL, 0.0, out)


def _tie(a, b):
    """Share of the gradient of min(a, b) that goes to a (torch.minimum's convention)."""

    return np.where(a < b, 1.0, np.where(a == b, 0.5, 0.0))


@dataclass
class PolicyCache:
    raw: dict
    mask: np.ndarray
    T: int
    z: np.ndarray = field(default=None)
    parts: dict = field(default_factory=dict)


def policy_forward(raw: dict, mask: np.ndarray) -> tuple[np.ndarray, PolicyCache]:
    """policy.py:113-204 in float64.  raw fields [S, W, ...]; mask [S, E] -> p [S, W, E]."""

    t = raw["type_logits"].astype(np.float64)
    om = raw["omega"].astype(np.float64)
    mu = raw["mu"].astype(np.float64)
    sc = raw["s"].astype(np.float64)
    io = raw["iota"].astype(np.float64)
    S, W, M = om.shape
    E = mask.shape[1]
    T = E - 2
    edges = np.linspace(0.0, 1.0, T + 1)
    z = (edges - mu[..., None]) / sc[..., None]  # [S,W,M,T+1]
    L, U = z[..., :-1], z[..., 1:]
    sU, snL, F = _sig(U), _sig(-L), -np.expm1(L - U)
    c = sU * snL * F
    c = np.where(np.abs(c) < SUBNORMAL, 0.0, c)
    b = np.maximum(c, 0.0)
    z0, zT = z[..., 0], z[..., -1]
    sT, sn0, FN = _sig(zT), _sig(-z0), -np.expm1(z0 - zT)
    N = sT * sn0 * FN
    Nc = np.maximum(N, TINY)
    a = b / Nc[..., None]
    Ssum = a.sum(-1)
    Sc = np.maximum(Ssum, TINY)
    dl = a / Sc[..., None]
    mix = (om[..., None] * dl).sum(-2)  # [S,W,T]
    rmask = np.broadcast_to(mask[:, None, 2:], (S, W, T))
    mixm = np.where(rmask, mix, 0.0)
    mass = mixm.sum(-1)
    cnt = rmask.sum(-1)
    uniform = rmask / np.maximum(cnt, 1)[..., None]
    pos = mass > 0
    cond = np.where(pos[..., None], mixm / np.maximum(mass, EPS)[..., None], uniform)
    idx = np.where(rmask, np.arange(T), -1).max(-1)
    allin = ((np.arange(T) == idx[..., None]) & (idx >= 0)[..., None]).astype(np.float64)
    rp = np.where(rmask, (1.0 - io[..., None]) * cond + io[..., None] * allin, 0.0)
    facing = np.broadcast_to(mask[:, None, 0], (S, W))
    x = np.empty((S, W, E))
    x[..., 0] = t[..., 0]
    x[..., 1] = np.where(facing, t[..., 1], t[..., 0])
    with np.errstate(divide="ignore"):
        x[..., 2:] = t[..., 2, None] + np.where(rp > 0, np.log(np.maximum(rp, EPS)), -np.inf)
    full_mask = np.broadcast_to(mask[:, None, :], (S, W, E))
    x = np.where(full_mask, x, -np.inf)
    mx = x.max(-1, keepdims=True)
    ex = np.where(full_mask, np.exp(x - mx), 0.0)
    p = ex / ex.sum(-1, keepdims=True)
    cache = PolicyCache(raw, mask, T, z)
    cache.parts = dict(om=om, mu=mu, sc=sc, io=io, sU=sU, snL=snL, F=F, c=c, b=b, sT=sT, sn0=sn0, FN=FN, N=N,
                       Nc=Nc, a=a, Ssum=Ssum, Sc=Sc, dl=dl, mixm=mixm, mass=mass, cond=cond, allin=allin, rp=rp,
                       rmask=rmask, facing=facing, full_mask=full_mask, p=p, L=L, U=U, z0=z0, zT=zT)
    return p, cache


def policy_backward(cache: PolicyCache, gp: np.ndarray, magnitude: bool = False) -> dict:
    """Gradient of the raw fields given dL/dp [S, W, E] (p after the masked fill).

    With ``magnitude`` the result is instead, per field, the sum of the
    absolute values of the terms the gradient is summed from, with every
    intermediate difference of the mixture chain (d mixture, d tick mass)
    replaced by the sum of its terms' absolute values.
    """

    P = cache.parts
    p, fm = P["p"], P["full_mask"]
    g = np.where(fm, gp, 0.0)
    dx = p * (g - (g * p).sum(-1, keepdims=True))  # softmax backward
    dx = np.where(fm, dx, 0.0)
    facing = P["facing"]
    S, W, E = p.shape
    A = np.abs if magnitude else (lambda v: v)
    dt = np.zeros((S, W, 3))
    dt[..., 0] = A(dx[..., 0]) + np.where(facing, 0.0, A(dx[..., 1]))
    dt[..., 1] = np.where(facing, A(dx[..., 1]), 0.0)
    dt[..., 2] = A(dx[..., 2:]).sum(-1)
    rp = P["rp"]
    drp = np.where(rp > 0, dx[..., 2:] * (rp >= EPS) / np.maximum(rp, EPS), 0.0)
    drp = np.where(P["rmask"], drp, 0.0)
    io = P["io"]
    dio = A(drp * (P["allin"] - P["cond"])).sum(-1)
    dcond = drp * (1.0 - io[..., None])
    mass, mixm = P["mass"], P["mixm"]
    pos = mass > 0
    mc = np.maximum(mass, EPS)
    dmass = -(mass >= EPS).astype(np.float64) * (dcond * mixm).sum(-1) / mc ** 2
    if magnitude:
        dmass = (mass >= EPS).astype(np.float64) * np.abs(dcond * mixm).sum(-1) / mc ** 2
        dmix = np.where(pos[..., None], np.abs(dcond) / mc[..., None] + dmass[..., None], 0.0)
    else:
        dmix = np.where(pos[..., None], dcond / mc[..., None] + dmass[..., None], 0.0)
    dmix = np.where(P["rmask"], dmix, 0.0)
    sgn = 1.0 if magnitude else -1.0  # the sign of every subtracted term below
    om, dl = P["om"], P["dl"]
    dom = (dmix[..., None, :] * dl).sum(-1)
    ddl = dmix[..., None, :] * om[..., None]
    Sc, Ssum, a = P["Sc"], P["Ssum"], P["a"]
    Q = (ddl * a).sum(-1)
    da = ddl / Sc[..., None] + sgn * ((Ssum >= TINY) * Q / Sc ** 2)[..., None]
    Nc, N, b = P["Nc"], P["N"], P["b"]
    db = da / Nc[..., None]
    dN = sgn * (N >= TINY).astype(np.float64) * (da * b).sum(-1) / Nc ** 2
    dc = db * (P["c"] >= 0)
    sU, snL, F = P["sU"], P["snL"], P["F"]
    # c = sig(U) sig(-L) F(L - U), F = -expm1(L - U): the product-rule terms of autograd
    ex = 1.0 - F  # exp(L - U)
    dU = dc * (sU * (1 - sU) * snL * F + sU * snL * ex)
    dL = sgn * dc * (sU * snL * (1 - snL) * F + sU * snL * ex)
    dz = np.zeros_like(cache.z)
    dz[..., 1:] += dU
    dz[..., :-1] += dL
    sT, sn0, FN = P["sT"], P["sn0"], P["FN"]
    exN = 1.0 - FN
    dz[..., -1] += dN * (sT * (1 - sT) * sn0 * FN + sT * sn0 * exN)
    dz[..., 0] += sgn * dN * (sT * sn0 * (1 - sn0) * FN + sT * sn0 * exN)
    sc = P["sc"]
    dmu = sgn * dz.sum(-1) / sc
    ds = sgn * (dz * A(cache.z)).sum(-1) / sc
    out = {"type_logits": dt, "omega": dom, "mu": dmu, "s": ds, "iota": dio}
    if magnitude:
        out = {k: np.abs(v) for k, v in out.items()}
    return out


@dataclass
class LearnerBatch:
    """One physical batch as forward_loss sees it (numpy, any float dtype)."""

    raw: dict                 # [S, W, ...]
    mask: np.ndarray          # [S, E] bool
    action_ptr: np.ndarray    # [S + 1]
    action: np.ndarray        # [A]
    old: np.ndarray           # [A, W]
    adv: np.ndarray           # [A, W]
    post: np.ndarray          # [A, W]
    value: np.ndarray         # [S, W]
    old_value: np.ndarray     # [S, W]
    target: np.ndarray        # [S, W]
    controls: np.ndarray      # [lanes, 10]
    lane_weight: np.ndarray   # [lanes]
    ref_raw: dict | None = None
    trace_pred: np.ndarray | None = None   # [S] (branched public heads)
    cost_pred: np.ndarray | None = None
    trace_target: np.ndarray | None = None
    cost_target: np.ndarray | None = None


def poker_learner_objective(batch: LearnerBatch, magnitude: bool = False):
    """learner.py:1824-2159 + the backward of (total * lane_weight).sum().

    Returns (result [lanes, 10] in ``RESULT`` order, grads dict with the raw
    fields, ``value`` and, for public heads, ``trace_pred`` / ``cost_pred``),
    plus, with ``magnitude``, a third dict with the raw-field gradient
    magnitudes (see ``policy_backward``).
    """

    p, cache = policy_forward(batch.raw, batch.mask)
    S, W, E = p.shape
    ptr = batch.action_ptr.astype(np.int64)
    counts = ptr[1:] - ptr[:-1]
    a2s = np.repeat(np.arange(S), counts)
    A = a2s.size
    lanes = batch.controls.shape[0]
    ctl = batch.controls.astype(np.float64)
    lw = batch.lane_weight.astype(np.float64)
    rpl = S // lanes
    apl = A // lanes
    sig_lane = np.arange(S) // rpl
    act_lane = np.arange(A) // apl
    logp = np.log(np.maximum(p, EPS))
    ent = -(p * logp).sum(-1)  # [S, W]
    if batch.ref_raw is not None:
        q, _ = policy_forward(batch.ref_raw, batch.mask)
        logq = np.log(np.maximum(q, EPS))
        kl = (p * (logp - logq)).sum(-1)
    else:
        logq = None
        kl = np.zeros((S, W))
    act = batch.action.astype(np.int64)
    pa = p[a2s, :, act]  # [A, W]
    cur = np.log(np.maximum(pa, EPS))
    old = batch.old.astype(np.float64)
    adv = batch.adv.astype(np.float64)
    post = batch.post.astype(np.float64)
    post = post / np.maximum(post.sum(-1, keepdims=True), TINY)
    lr = cur - old
    ratio = np.exp(lr)
    clip = ctl[act_lane, 0][:, None]
    cap = ctl[act_lane, 1][:, None]
    clipped = np.clip(ratio, 1 - clip, 1 + clip)
    neg = adv < 0
    lr_capped = np.minimum(lr, cap)
    nratio = np.exp(lr_capped)
    pratio = np.where(neg, nratio, ratio)
    neg_capped = neg & (lr > cap)
    X, Y = pratio * adv, clipped * adv
    term = -np.minimum(X, Y)
    policy_row = (post * term).sum(-1)
    entropy_row = (post * ent[a2s]).sum(-1)
    reference_row = (post * kl[a2s]).sum(-1)
    approx_row = (post * ((ratio - 1) - lr)).sum(-1)
    clipped_row = (post * (np.abs(ratio - 1) > clip)).sum(-1)
    negcap_row = (post * neg_capped).sum(-1)
    sup_neg = neg & (post > 0)
    nlr_max = np.full(lanes, -np.inf)
    ninf_max = np.full(lanes, -np.inf)
    nlr_vals = np.where(sup_neg, lr, 0.0)
    ninf_vals = post * np.maximum(-adv, 0.0) * np.where(neg, pratio, 0.0)
    for ln in range(lanes):
        sl = act_lane == ln
        nlr_max[ln] = nlr_vals[sl].max()
        ninf_max[ln] = ninf_vals[sl].max()
    sigma_post = np.zeros((S, W))
    np.add.at(sigma_post, a2s, post)
    sigma_post /= counts[:, None]
    sigma_post /= np.maximum(sigma_post.sum(-1, keepdims=True), TINY)
    v = batch.value.astype(np.float64)
    ov = batch.old_value.astype(np.float64)
    tg = batch.target.astype(np.float64)
    veps = ctl[sig_lane, 3][:, None]
    use_clip = ctl[sig_lane, 9][:, None] != 0
    verr = (v - tg) ** 2
    diff = v - ov
    cv = ov + np.clip(diff, -veps, veps)
    cerr = (cv - tg) ** 2
    value_error = np.where(use_clip, np.maximum(verr, cerr), verr)
    value_row = (sigma_post * value_error).sum(-1)

    def mean_by_sigma(rows):
        out = np.zeros(S)
        np.add.at(out, a2s, rows)
        return out / counts

    def lane_mean(vals):
        return vals.reshape(lanes, -1).mean(-1)

    sig_policy = mean_by_sigma(policy_row)
    branched_heads = batch.trace_pred is not None
    if branched_heads:
        e8 = ctl[sig_lane, 8]
        tp = batch.trace_pred.astype(np.float64)
        cp = batch.cost_pred.astype(np.float64)
        tt = batch.trace_target.astype(np.float64)
        ct = batch.cost_target.astype(np.float64)
        tr = (tt + e8) / (np.maximum(tp, TINY) + e8)
        trace_terms = np.where(counts >= 2, tr - np.log(tr) - 1, 0.0)
        cr = ct / np.maximum(cp, TINY)
        cost_terms = cr - np.log(cr) - 1
        trace_loss, cost_loss = lane_mean(trace_terms), lane_mean(cost_terms)
    else:
        trace_loss = cost_loss = np.zeros(lanes)
    policy_loss = lane_mean(sig_policy)
    value_loss = lane_mean(value_row)
    entropy_mean = lane_mean(mean_by_sigma(entropy_row))
    ref_mean = lane_mean(mean_by_sigma(reference_row))
    total = (policy_loss + ctl[:, 2] * value_loss - ctl[:, 4] * entropy_mean + ctl[:, 5] * ref_mean
             + ctl[:, 6] * trace_loss + ctl[:, 7] * cost_loss)
    result = np.stack([total, policy_loss, value_loss, entropy_mean, ref_mean,
                       lane_mean(mean_by_sigma(approx_row)), lane_mean(mean_by_sigma(clipped_row)),
                       lane_mean(mean_by_sigma(negcap_row)), nlr_max, ninf_max], 1)

    # ---- backward of sum_l lw_l * total_l
    row_scale = (lw[act_lane] / rpl / counts[a2s])[:, None]          # d total / d policy_row_i
    gx, gy = _tie(X, Y), _tie(Y, X)
    dpr = np.where(neg, nratio * _tie(lr, cap), ratio)
    dclip = ratio * ((ratio >= 1 - clip) & (ratio <= 1 + clip))
    dcur = -row_scale * post * (gx * adv * dpr + gy * adv * dclip)  # [A, W]
    dpa = dcur * (pa >= EPS) / np.maximum(pa, EPS)
    gp = np.zeros((S, W, E))
    np.add.at(gp, (a2s, slice(None), act), dpa)
    # entropy and KL rows: coefficient per (s, c) = sum over the span of post / count
    wsum = np.zeros((S, W))
    np.add.at(wsum, a2s, post * row_scale)
    ge = ctl[sig_lane, 4][:, None] * wsum   # d total / d entropy_{s,c} = -c4 * wsum
    gk = ctl[sig_lane, 5][:, None] * wsum
    ind = (p >= EPS).astype(np.float64)
    gp += -ge[..., None] * (-logp - ind)
    if logq is not None:
        gp += gk[..., None] * (logp - logq + ind)
    grads = policy_backward(cache, gp)
    mags = policy_backward(cache, gp, magnitude=True) if magnitude else None
    # value
    vscale = (ctl[sig_lane, 2] * lw[sig_lane] / rpl)[:, None] * sigma_post
    dverr = 2 * (v - tg)
    dcerr = 2 * (cv - tg) * ((diff >= -veps) & (diff <= veps))
    dvalue = np.where(use_clip, _tie(cerr, verr) * dverr + _tie(verr, cerr) * dcerr, dverr)
    grads["value"] = vscale * dvalue
    if branched_heads:
        hs = lw[sig_lane] / rpl
        dtr = np.where(counts >= 2, 1 - 1 / tr, 0.0)
        grads["trace_pred"] = ctl[sig_lane, 6] * hs * dtr * (-(tt + e8) / (np.maximum(tp, TINY) + e8) ** 2) \
            * (tp >= TINY)
        grads["cost_pred"] = ctl[sig_lane, 7] * hs * (1 - 1 / cr) * (-ct / np.maximum(cp, TINY) ** 2) * (cp >= TINY)
    if magnitude:
        return result, grads, mags
    return result, grads


def policy_learner_vjp(raw: dict, ref_raw: dict | None, mask: np.ndarray, action: np.ndarray, g_sel, g_ent, g_kl,
                       magnitude: bool = False):
    """PokerPolicyOperator.learner (policy.py:284-298): forward values and the raw-field gradient of
    sum(g_sel * selected + g_ent * entropy + g_kl * kl) for policy rows [B, rows]."""

    p, cache = policy_forward(raw, mask)
    B, rows, E = p.shape
    logp = np.log(np.maximum(p, EPS))
    act = action.astype(np.int64)
    pa = p[np.arange(B), :, act]
    sel = np.log(np.maximum(pa, EPS))
    ent = -(p * logp).sum(-1)
    ind = (p >= EPS).astype(np.float64)
    gp = np.zeros_like(p)
    gp[np.arange(B), :, act] = np.asarray(g_sel, np.float64) * (pa >= EPS) / np.maximum(pa, EPS)
    gp += np.asarray(g_ent, np.float64)[..., None] * -(logp + ind)
    kl = np.zeros((B, rows))
    if ref_raw is not None:
        q, _ = policy_forward(ref_raw, mask)
        logq = np.log(np.maximum(q, EPS))
        kl = (p * (logp - logq)).sum(-1)
        gp += np.asarray(g_kl, np.float64)[..., None] * (logp - logq + ind)
    grads = policy_backward(cache, gp)
    if magnitude:
        return (sel, ent, kl), grads, policy_backward(cache, gp, magnitude=True)
    return (sel, ent, kl), grads


def within_rounding(got, want, mag, *, atol=2e-6, rtol=2e-5, k=16.0):
    """Elementwise |got - want| <= atol + rtol |want| + k 2^-24 mag (see the module docstring)."""

    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    bound = atol + rtol * np.abs(want) + k * 2.0 ** -24 * np.asarray(mag, np.float64)
    return np.abs(got - want) <= bound


def from_golden(d: dict, name: str) -> LearnerBatch:
    """The inputs of one golden case (tests/golden/poker_loss.npz) as a LearnerBatch."""

    pre = f"pl_{name}_"
    raw = {k: d[pre + k] for k in FIELDS}
    ref = {k: d[pre + "ref_" + k] for k in FIELDS} if (pre + "ref_mu") in d else None
    kw = {}
    if (pre + "trace_pred") in d:
        kw = dict(trace_pred=d[pre + "trace_pred"], cost_pred=d[pre + "cost_pred"],
                  trace_target=d[pre + "trace_target"], cost_target=d[pre + "cost_target"])
    return LearnerBatch(raw, d[pre + "mask"].astype(bool), d[pre + "action_ptr"], d[pre + "action"], d[pre + "old"],
                        d[pre + "adv"], d[pre + "post"], d[pre + "value"], d[pre + "old_value"], d[pre + "target"],
                        d[pre + "controls"], d[pre + "lane_weight"], ref, **kw)


def seeded_batch(seed: int, *, S: int, W: int, E: int, M: int = 2, lanes: int = 1, max_span: int = 1,
                 reference: bool = True, heads: bool = False, masks: np.ndarray | None = None) -> LearnerBatch:
    """A synthetic physical batch with the value distributions of the golden cases."""

    rng = np.random.default_rng(seed)
    f32 = np.float32
    logits = (rng.standard_normal((S, W, 3)) * 1.5).astype(f32)
    w = rng.standard_normal((S, W, M))
    om = np.exp(w - w.max(-1, keepdims=True))
    om = (om / om.sum(-1, keepdims=True)).astype(f32)
    mu = (1 / (1 + np.exp(-rng.standard_normal((S, W, M))))).astype(f32)
    sc = (np.log1p(np.exp(rng.standard_normal((S, W, M)))) + 0.02).astype(f32)
    io = (1 / (1 + np.exp(-rng.standard_normal((S, W))))).astype(f32)
    raw = {"type_logits": logits, "omega": om, "mu": mu, "s": sc, "iota": io}
    ref = None
    if reference:
        ref = {k: v.copy() for k, v in raw.items()}
        ref["type_logits"] = (ref["type_logits"] + 0.3 * rng.standard_normal((S, W, 3))).astype(f32)
        ref["mu"] = np.clip(ref["mu"] + 0.1 * rng.standard_normal((S, W, M)), 0, 1).astype(f32)
    if masks is None:
        mask = rng.random((S, E)) < 0.6
        mask[:, 1] = True
    else:
        mask = masks[rng.integers(0, masks.shape[0], S)]
    if max_span > 1:
        per_lane = S // lanes
        base = rng.integers(1, max_span + 1, per_lane)
        counts = np.tile(base, lanes)
    else:
        counts = np.ones(S, np.int64)
    ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    A = int(counts.sum())
    a2s = np.repeat(np.arange(S), counts)
    action = np.array([rng.choice(np.nonzero(mask[s])[0]) for s in a2s], dtype=np.int32)
    p, _ = policy_forward(raw, mask)
    cur = np.log(np.maximum(p[a2s, :, action], EPS))
    old = (cur + 0.3 * rng.standard_normal((A, W))).astype(f32)
    far = rng.random(A) < 0.3
    old[far] += (1.5 * rng.standard_normal((int(far.sum()), W))).astype(f32)
    adv = rng.standard_normal((A, W)).astype(f32)
    if W > 1:
        post = (rng.random((A, W)) * (rng.random((A, W)) > 0.3)).astype(f32)
    else:
        post = np.ones((A, 1), f32)
    value = rng.standard_normal((S, W)).astype(f32)
    old_value = (value + 0.3 * rng.standard_normal((S, W))).astype(f32)
    target = rng.standard_normal((S, W)).astype(f32)
    base_ctl = [[0.2, math.log(1.5), 0.5, 0.2, 0.01, 0.05 if reference else 0.0, 0.3 if heads else 0.0,
                 0.2 if heads else 0.0, 1e-3 if heads else 1e-8, 1.0],
                [0.25, math.inf, 0.7, 0.0, 0.02, 0.1 if reference else 0.0, 0.1 if heads else 0.0,
                 0.4 if heads else 0.0, 1e-2 if heads else 1e-8, 0.0]]
    controls = np.array([base_ctl[i % 2] for i in range(lanes)], dtype=f32)
    lane_weight = np.array([(1.6, 0.5, 1.0, 0.25)[i % 4] for i in range(lanes)], dtype=f32)
    kw = {}
    if heads:
        kw = dict(trace_pred=(rng.random(S) * 2 + 0.05).astype(f32), cost_pred=(rng.random(S) * 2 + 0.05).astype(f32),
                  trace_target=(rng.random(S) * 2).astype(f32), cost_target=(rng.random(S) * 2 + 0.01).astype(f32))
    return LearnerBatch(raw, mask, ptr, action, old, adv, post, value, old_value, target, controls, lane_weight,
                        ref, **kw)
