"""The network's backward (pbg_b200.model_train) against torch fp32 autograd and the reference's own
gradients.

Op level: each autograd function of the training forward (dense map with GELU / residual / row
scale epilogues, LayerNorm, reach-biased attention with absent keys and a sequence without keys)
against torch fp32 autograd of the same op on the same bf16-rounded operands; tolerance the bf16
bar, 2e-2 of the reference's largest magnitude.

Network level: tests/golden/{pre,post}flop_model*.npz hold, beside the reference modules' outputs,
the reference's own autograd gradient of a seeded loss sum_f <c_f, output_f> with respect to every
parameter (run on CPU by tests/golden/make_golden.py), sketched per parameter by its norm and its
projections onto seeded probe vectors (tests/golden/model_params.py probe).  This build's training
forward and backward on the same weights and inputs must give, per parameter, a relative gradient
error sqrt(mean((proj - proj_ref)^2)) / |g_ref| (an estimate of |g - g_ref| / |g_ref|) below 5e-2
and a norm within 5e-2, the bf16 bar for gradients through two bf16 passes.
"""

import os
import sys

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def _bf(t):
    return t.to(torch.bfloat16).float()


def _close(got, ref, tol=2e-2):
    scale = float(ref.abs().max()) + 1e-12
    err = float((got.float() - ref).abs().max())
    assert err <= tol * scale, f"max error {err:.3e} vs scale {scale:.3e}"


@pytest.mark.parametrize("activation,group,scaled,out_dtype", [
    (None, 1, False, torch.float32), ("gelu", 1, False, torch.float32), ("gelu", 4, False, torch.float32),
    (None, 1, True, torch.float32), ("gelu", 1, False, torch.bfloat16), ("gelu", 4, True, torch.bfloat16)])
def test_linear_backward_matches_torch(activation, group, scaled, out_dtype):
    """bf16 outputs of a GELU map take the fused path (pbg_linear_gelu_backward: the pre-activation
    recomputed with dy * GELU' in the epilogue); fp32 outputs the recompute + pbg_gelu_backward path."""

    from pbg_b200.preflop import _Binding, _Map, _padded

    g = torch.Generator(device=DEV).manual_seed(3)
    M, K, Nn = 512, 200, 256
    w = (torch.randn(Nn, K, device=DEV, generator=g) / K ** 0.5).requires_grad_()
    b = (torch.randn(Nn, device=DEV, generator=g) * 0.1).requires_grad_()
    x = torch.randn(M, K, device=DEV, generator=g).requires_grad_()
    res = torch.randn(M // group, Nn, device=DEV, generator=g).requires_grad_()
    scale = torch.rand(M, device=DEV, generator=g) + 0.5 if scaled else None
    binding = _Binding()
    binding.training = True
    m = _Map(w, b, DEV, source=lambda: (w, b), binding=binding)
    y = m.apply(_padded(x, m.kp), activation, row_scale=scale, residual=res, residual_group=group,
                out_dtype=out_dtype)
    c = torch.randn(M, Nn, device=DEV, generator=g)
    (y.float() * c).sum().backward()
    got = [t.grad.clone() for t in (x, w, b, res)]
    for t in (x, w, b, res):
        t.grad = None
    pre = _bf(x) @ _bf(w).t()
    if scaled:
        pre = pre * scale[:, None]
    pre = pre + b + res.repeat_interleave(group, 0)
    ref = F.gelu(pre) if activation == "gelu" else pre
    (ref * (c if out_dtype == torch.float32 else _bf(c))).sum().backward()
    for a, t in zip(got, (x, w, b, res)):
        _close(a, t.grad)


def test_layernorm_backward_matches_torch():
    from pbg_b200.model_train import layernorm_train

    g = torch.Generator(device=DEV).manual_seed(4)
    for d in (128, 256):
        x = (torch.randn(3000, d, device=DEV, generator=g) * 2 + 0.5).requires_grad_()
        gain = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).requires_grad_()
        bias = (0.1 * torch.randn(d, device=DEV, generator=g)).requires_grad_()
        c = torch.randn(3000, d, device=DEV, generator=g)
        (layernorm_train(x, gain, bias).float() * c).sum().backward()
        got = [t.grad.clone() for t in (x, gain, bias)]
        for t in (x, gain, bias):
            t.grad = None
        (F.layer_norm(x, (d,), gain, bias, 1e-5) * _bf(c)).sum().backward()
        for a, t in zip(got, (x, gain, bias)):
            _close(a, t.grad)


@pytest.mark.parametrize("length", [200, 700])
def test_attention_backward_matches_torch(length):
    from pbg_b200.model_train import attention_train, q_scale_of

    g = torch.Generator(device=DEV).manual_seed(5)
    B, H = 3, 4
    qkv = (torch.randn(B, length, 3 * H * 32, device=DEV, generator=g)).to(torch.bfloat16).requires_grad_()
    theta = torch.randn(H, device=DEV, generator=g).mul(0.1).add(-0.5).requires_grad_()
    bias = torch.randn(B, length, device=DEV, generator=g)
    mask = torch.rand(B, length, device=DEV, generator=g) < 0.8
    mask[2] = False  # a sequence without keys: its outputs and gradients are zero
    out = attention_train(qkv, H, q_scale_of(theta), bias, mask)
    c = torch.randn(B, length, H * 32, device=DEV, generator=g)
    (out.float() * c).sum().backward()
    got_qkv, got_theta = qkv.grad.float().clone(), theta.grad.clone()
    qkv.grad, theta.grad = None, None
    x = qkv.float().view(B, length, 3, H, 32)
    q, k, v = (x[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    scores = torch.einsum("bhid,bhjd->bhij", q, k) * q_scale_of(theta)[None, :, None, None] + bias[:, None, None]
    scores = scores.masked_fill(~mask[:, None, None], -torch.inf)
    p = torch.nan_to_num(torch.softmax(scores, -1), nan=0.0)
    ref = torch.einsum("bhij,bhjd->bhid", p, v).permute(0, 2, 1, 3).reshape(B, length, H * 32)
    _close(out.float().detach(), ref.detach())
    (ref * _bf(c)).sum().backward()
    _close(got_qkv, qkv.grad.float())
    _close(got_theta, theta.grad)
    assert float(got_qkv[2].abs().max()) == 0.0


@pytest.mark.parametrize("players,rows,shared_scale", [(2, 169, True), (3, 300, False)])
def test_incidence_combine_backward_matches_torch(players, rows, shared_scale):
    """incidence.py:57-70 seat sums: [oe | own], oc and [oc^2 | oc oe] and their backward against torch fp32
    autograd of the same formulas (bf16 outputs rounded as the kernel's)."""

    from pbg_b200.model_train import incidence_combine_train

    g = torch.Generator(device=DEV).manual_seed(6)
    B, d = 4, 128
    source = torch.randn(B, players, rows, d, device=DEV, generator=g).requires_grad_()
    overlap = torch.randn(B, players, rows, d, device=DEV, generator=g).requires_grad_()
    scale = (torch.rand(rows, device=DEV, generator=g) + 0.1)[None].expand(B, -1) if shared_scale else \
        torch.ones(B, rows, device=DEV)
    pair, oc, feats = incidence_combine_train(source, overlap, scale)
    c1, c2, c3 = (torch.randn(t.shape, device=DEV, generator=g) for t in (pair, oc, feats))
    ((pair.float() * c1).sum() + (oc * c2).sum() + (feats.float() * c3).sum()).backward()
    got = [source.grad.clone(), overlap.grad.clone()]
    source.grad, overlap.grad = None, None
    same = source * scale[:, None, :, None]
    oe = same.sum(1, keepdim=True) - same
    occ = (overlap.sum(1, keepdim=True) - overlap) - 2.0 * oe
    own = overlap - 2.0 * same
    count = B * players * rows
    ref_pair = torch.cat((oe.reshape(count, d), own.reshape(count, d)), -1)
    ref_feats = torch.cat(((occ * occ).reshape(count, d), (occ * oe).reshape(count, d)), -1)
    _close(pair.float().detach(), ref_pair.detach())
    _close(oc.detach(), occ.reshape(count, d).detach(), tol=1e-5)
    _close(feats.float().detach(), ref_feats.detach())
    ((ref_pair * _bf(c1)).sum() + (occ.reshape(count, d) * c2).sum() + (ref_feats * _bf(c3)).sum()).backward()
    _close(got[0], source.grad, tol=1e-4)
    _close(got[1], overlap.grad, tol=1e-4)


def _sketch_check(model_params, d, leaves):
    names = [str(n) for n in d["gsk_names"]]
    norms, projections = d["gsk_norm"], d["gsk_proj"]
    top = float(norms.max())
    worst = []
    for i, name in enumerate(names):
        grad = leaves[name].grad
        flat = grad.detach().reshape(-1).double().cpu().numpy()
        ref = float(norms[i])
        if ref <= 1e-7 * top:
            assert float(np.abs(flat).max()) <= 1e-6 * top, f"{name}: gradient where the reference has none"
            continue
        proj = model_params.probe(name, tuple(grad.shape)) @ flat
        rel = float(np.sqrt(np.mean((proj - projections[i]) ** 2))) / ref
        worst.append((rel, abs(float(np.linalg.norm(flat)) / ref - 1.0), name))
    worst.sort(reverse=True)
    print("\nworst relative gradient errors:", [(f"{r:.3e}", f"{n:.3e}", name) for r, n, name in worst[:6]])
    for rel, norm_err, name in worst:
        assert rel < 5e-2 and norm_err < 5e-2, f"{name}: relative error {rel:.3e}, norm error {norm_err:.3e}"


def _train(model):
    from pbg_b200.model_train import FlatParameters

    flat = FlatParameters(model.p, DEV)
    model.bind_parameters(flat.leaves)
    model.train()
    flat.attach(torch.zeros(flat.numel, dtype=torch.float32, device=DEV))
    return flat


def _seeded_loss(d, raw, value):
    loss = sum((torch.from_numpy(d["gcoef_" + k]).to(DEV) * raw[k]).sum() for k in raw)
    return loss + (torch.from_numpy(d["gcoef_value"]).to(DEV) * value).sum()


@pytest.mark.parametrize("fixture", ["preflop_model", "preflop_model_r13"])
def test_preflop_gradients_match_reference_autograd(gold, fixture):
    import model_params
    from test_gpu_preflop import _model, _pub

    d = gold(fixture)
    model, _ = _model(d)
    flat = _train(model)
    raw, value = model.forward(_pub(d), torch.from_numpy(d["class_ranges"]).to(DEV),
                               torch.from_numpy(d["class_mask"]).to(DEV))
    for k in raw:  # the training forward computes what the inference forward does
        torch.testing.assert_close(raw[k].detach().cpu(), torch.from_numpy(d["raw_" + k]), rtol=2e-2, atol=2e-2)
    _seeded_loss(d, raw, value).backward()
    torch.cuda.synchronize()
    _sketch_check(model_params, d, flat.leaves)


@pytest.mark.parametrize("fixture", ["postflop_model", "postflop_model_r13"])
def test_postflop_gradients_match_reference_autograd(gold, fixture):
    import model_params
    from test_gpu_postflop import _inputs, _model, _params

    d = gold(fixture)
    model = _model(_params(d), d)
    flat = _train(model)
    pub, ranges, masks = _inputs(d)
    raw, value = model.forward(pub, ranges, None, masks)
    for k in raw:
        torch.testing.assert_close(raw[k].detach().cpu(), torch.from_numpy(d["raw_" + k]), rtol=2e-2, atol=2e-2)
    _seeded_loss(d, raw, value).backward()
    torch.cuda.synchronize()
    _sketch_check(model_params, d, flat.leaves)


def test_inference_after_training_mode_uses_updated_weights(gold):
    """train(False) refreshes every map from the parameters: a changed weight changes the outputs."""

    from test_gpu_preflop import _model, _pub

    d = gold("preflop_model")
    model, _ = _model(d)
    flat = _train(model)
    with torch.no_grad():
        flat.leaves["layer_ffns.1.output.weight"].mul_(1.5)
    model.train(False)
    raw, _ = model.forward(_pub(d), torch.from_numpy(d["class_ranges"]).to(DEV),
                           torch.from_numpy(d["class_mask"]).to(DEV))
    assert float((raw["type_logits"].cpu() - torch.from_numpy(d["raw_type_logits"])).abs().max()) > 5e-2


def test_queued_learner_gradients_match_reference_autograd(gold):
    """The learner rows of every partition of the queued model (3-handed R4, branching heads on): one
    seeded loss over the pre, post_2 and post_3 learner outputs, the shared parameters collecting the
    gradient of both networks, against the reference QueuedPokerModel's own autograd."""

    import model_params
    from test_gpu_queued_model import _model

    d = gold("queued_model")
    model = _model(d)
    flat = model.enable_training()
    flat.attach(torch.zeros(flat.numel, dtype=torch.float32, device=DEV))
    loss = 0.0
    for kind in [str(x) for x in d["partitions"]]:
        tag = "q_" + kind
        rows = torch.from_numpy(d[tag + "_model_input"]).to(DEV)
        private = torch.from_numpy(d[tag + "_private"]).to(DEV)
        owner = model._state(kind, rows).to_act.to(torch.int64)
        result = model.learner_operation(kind, rows, private, owner)
        for name, value in result.policy_raw.items():
            torch.testing.assert_close(value.detach().cpu(), torch.from_numpy(d[tag + "_lraw_" + name]),
                                       rtol=2e-2, atol=2e-2)
            loss = loss + (torch.from_numpy(d[f"gcoef_{kind}__{name}"]).to(DEV) * value).sum()
        loss = loss + (torch.from_numpy(d[f"gcoef_{kind}__value"]).to(DEV) * result.value).sum()
    loss.backward()
    torch.cuda.synchronize()
    _sketch_check(model_params, d, flat.leaves)


def _learner_batch(model, d, kind, seed):
    """The fixture's learner rows of one partition with a seeded objective batch (legal taken actions)."""

    g = torch.Generator(device=DEV).manual_seed(seed)
    tag = "q_" + kind
    rows = torch.from_numpy(d[tag + "_model_input"]).to(DEV)
    S, E = rows.shape[0], model.geometry.events
    mask = torch.zeros(S, E, dtype=torch.bool, device=DEV)
    mask[:, 1] = True
    mask[:, 0] = torch.rand(S, device=DEV, generator=g) < 0.7
    mask[:, 2:] = torch.rand(S, E - 2, device=DEV, generator=g) < 0.5
    pick = (torch.rand(S, device=DEV, generator=g) * mask.sum(1)).long()
    action = (mask.cumsum(1) <= pick[:, None]).sum(1).to(torch.int32)
    return {"input_type": kind, "model_input": rows, "sampled_private_state": torch.from_numpy(d[tag + "_private"]).to(DEV),
            "owner": model._state(kind, rows).to_act.to(torch.int64), "mask": mask, "action": action,
            "old_log_policy": -1.5 + 0.5 * torch.randn(S, 1, device=DEV, generator=g),
            "advantage_target": torch.randn(S, 1, device=DEV, generator=g),
            "old_value": torch.randn(S, 1, device=DEV, generator=g),
            "value_target": torch.randn(S, 1, device=DEV, generator=g),
            "controls": torch.tensor([[0.2, 0.405, 0.5, 0.2, 0.01, 0.05, 0.0, 0.0, 1e-8, 1.0]], device=DEV),
            "lane_weight": torch.ones(1, device=DEV)}


def test_model_learner_step_accumulates_families_and_steps(gold):
    """ModelLearnerStep: the flat gradient of a pre + post_2 step is the sum of the two families' own
    gradients (the shared parameters collect both), and the AdamW step moves the parameters."""

    from pbg_b200.model_train import ModelLearnerStep
    from test_gpu_queued_model import _model

    d = gold("queued_model")
    step = ModelLearnerStep(_model(d))
    model = step.model
    pre, post = _learner_batch(model, d, "pre", 1), _learner_batch(model, d, "post_2", 2)
    step.adam.grad.zero_()
    step.gradient([pre])
    g_pre = step.adam.grad.clone()
    step.adam.grad.zero_()
    step.gradient([post])
    g_post = step.adam.grad.clone()
    step.adam.grad.zero_()
    results = step.gradient([pre, post])
    both = step.adam.grad.clone()
    assert all(bool(torch.isfinite(r.total).all()) for r in results)
    assert float(g_pre.abs().max()) > 0 and float(g_post.abs().max()) > 0
    torch.testing.assert_close(both, g_pre + g_post, rtol=1e-4, atol=1e-6 * float(both.abs().max()))
    before = step.flat.master.clone()
    report = step.adam.step()
    torch.cuda.synchronize()
    assert bool(torch.isfinite(report).all())
    assert float((step.flat.master - before).abs().max()) > 0
    # each step's gradient starts from zero: the transition leaves the clipped gradient in the buffer
    step.adam.step()
    first = step.gradient([pre])
    g1 = step.adam.grad.clone()
    step.gradient([pre])
    torch.testing.assert_close(step.adam.grad, g1, rtol=1e-5, atol=1e-7 * float(g1.abs().max()))
    assert all(bool(torch.isfinite(r.total).all()) for r in first)
