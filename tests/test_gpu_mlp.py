"""The cfg1 preflop-class MLP and its learner step (pbg_b200.mlp) against a PyTorch restatement.

The reference has no MLP (its preflop model is a transformer); cfg1's MLP sits
behind the reference's ModelOperation protocol (pbg/core/learner.py:324-350)
with the reference heads' activations (pbg/games/poker/model/heads.py:28-62),
so its parity is to the same network written in torch: the forward within
1e-6, and the flat gradient of the fused objective within rtol 1e-4 of torch
autograd through the restated network (the dense maps are the same cuBLAS
GEMMs; the heads, epilogues and bias sums are this library's).
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _batch(geometry, S, seed=3, M=2):
    g = torch.Generator(device=DEV).manual_seed(seed)
    E = geometry.events
    T = E - 2
    mask = torch.zeros(S, E, dtype=torch.bool, device=DEV)
    mask[:, 1] = True
    mask[:, 0] = torch.rand(S, device=DEV, generator=g) < 0.7
    lo = torch.randint(0, T, (S,), device=DEV, generator=g)
    ticks = torch.arange(T, device=DEV)
    mask[:, 2:] = (torch.rand(S, device=DEV, generator=g) >= 0.1)[:, None] & (ticks[None] >= lo[:, None])
    pick = (torch.rand(S, device=DEV, generator=g) * mask.sum(1)).long()
    action = (mask.cumsum(1) <= pick[:, None]).sum(1).to(torch.int32)
    return {"model_input": torch.randn(S, geometry.preflop_model_input_width, device=DEV, generator=g),
            "sampled_class": torch.randint(0, geometry.private_classes, (S,), device=DEV, generator=g),
            "mask": mask, "action": action,
            "old_log_policy": -1.5 + 0.5 * torch.randn(S, 1, device=DEV, generator=g),
            "advantage_target": torch.randn(S, 1, device=DEV, generator=g),
            "old_value": torch.randn(S, 1, device=DEV, generator=g),
            "value_target": torch.randn(S, 1, device=DEV, generator=g),
            "controls": torch.tensor([[0.2, math.log(1.5), 0.5, 0.2, 0.01, 0.05, 0.0, 0.0, 1e-8, 1.0]], device=DEV),
            "lane_weight": torch.full((1,), 0.75, device=DEV)}


def torch_forward(model, params, x, cls):
    """The same network in torch ops (the bias added after each GEMM, as the library does)."""

    h1 = torch.relu(torch.mm(x, params["w1"].t()) + params["b1"])
    h2 = torch.relu(torch.mm(h1, params["w2"].t()) + params["b2"])
    z = torch.mm(h2, params["w3"].t()) + params["b3"]
    K, R, M = model.K, model.row, model.M
    rows = z[:, :K * R].reshape(-1, K, R)[torch.arange(x.shape[0], device=DEV), cls.long()]
    raw = {"type_logits": rows[:, None, :3], "omega": torch.softmax(rows[:, 3:3 + M], -1)[:, None],
           "mu": torch.sigmoid(rows[:, 3 + M:3 + 2 * M])[:, None],
           "s": (torch.nn.functional.softplus(rows[:, 3 + 2 * M:3 + 3 * M]) + model.s_min)[:, None],
           "iota": torch.sigmoid(rows[:, 3 + 3 * M])[:, None]}
    value = z[torch.arange(x.shape[0], device=DEV), K * R + cls.long()][:, None]
    return raw, value


@pytest.mark.parametrize("players,stack,ranks", [(2, 8.0, 4), (2, 100.0, 13)])
def test_mlp_forward_matches_torch(players, stack, ranks):
    from pbg_b200.mlp import PreflopMLP
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(players, stack, ranks)
    model = PreflopMLP(geometry, device=DEV, seed=1)
    b = _batch(geometry, 3000)
    raw, value, _ = model.forward(b["model_input"], b["sampled_class"])
    model.check()
    want_raw, want_value = torch_forward(model, model.params, b["model_input"], b["sampled_class"])
    for k, v in want_raw.items():
        torch.testing.assert_close(raw[k], v, rtol=1e-6, atol=1e-6, msg=k)
    torch.testing.assert_close(value, want_value, rtol=1e-6, atol=1e-6)
    bad = b["sampled_class"].clone()
    bad[7] = geometry.private_classes
    model.forward(b["model_input"], bad)
    with pytest.raises(ValueError):
        model.check()


@pytest.mark.parametrize("S", [1, 1000, 16384])
def test_mlp_gradient_matches_autograd(S):
    from pbg_b200.learner import poker_learner_loss
    from pbg_b200.mlp import MLPLearnerStep, PreflopMLP
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    model = PreflopMLP(geometry, device=DEV, seed=2)
    step = MLPLearnerStep(model)
    b = _batch(geometry, S, seed=S)
    result = step.gradient(b)
    got = step.adam.grad.clone()
    leaves = {k: v.detach().clone().requires_grad_() for k, v in model.params.items()}
    raw, value = torch_forward(model, leaves, b["model_input"], b["sampled_class"])
    loss = poker_learner_loss(None, raw, value, mask=b["mask"], action=b["action"],
                              old_log_policy=b["old_log_policy"], advantage_target=b["advantage_target"],
                              old_value=b["old_value"], value_target=b["value_target"], controls=b["controls"])
    (loss.total * b["lane_weight"]).sum().backward()
    want = torch.cat([leaves[name].grad.reshape(-1) for name, _ in model.shapes])
    scale = float(want.abs().max())
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5 * scale)
    torch.testing.assert_close(result.total, loss.total.detach(), rtol=1e-5, atol=1e-6)


def test_mlp_learner_step_is_deterministic_and_moves_the_model():
    from pbg_b200.mlp import MLPLearnerStep, PreflopMLP
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    finals = []
    for _ in range(2):
        model = PreflopMLP(geometry, device=DEV, seed=4)
        start = model.master.clone()
        step = MLPLearnerStep(model, lr=1e-3)
        for i in range(3):
            step(_batch(geometry, 4096, seed=10 + i))
        assert not torch.equal(model.master, start)
        finals.append(model.master.clone())
    assert torch.equal(finals[0], finals[1])
