"""Host logic of the network's training mode (pbg_b200.model_train, the training paths of
pbg_b200.preflop), on CPU: no kernel is launched.

- FlatParameters: every parameter a leaf view of one flat master, gradients accumulated in place in
  one flat buffer (shared leaves collect every use);
- lookup: the one-hot product used while a table takes a gradient equals plain indexing exactly, and
  its gradient equals the index scatter's;
- _padded: the training pad gives the same operand as the inference pad and a sliced gradient;
- FamilyModel.bind_parameters / sync_weights: the maps' fused weights follow the bound parameters.
"""

import math
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def test_flat_parameters_views_and_in_place_gradients():
    from pbg_b200.model_train import FlatParameters

    gen = torch.Generator().manual_seed(0)
    params = {"a": torch.randn(3, 4, generator=gen), "b": torch.randn(5, generator=gen),
              "c": torch.randn(2, 2, 2, generator=gen)}
    flat = FlatParameters(params, "cpu")
    assert flat.numel == 12 + 5 + 8 and flat.names == ["a", "b", "c"]
    grad = torch.zeros(flat.numel)
    flat.attach(grad)
    for name, value in params.items():
        leaf = flat.leaves[name]
        assert leaf.is_leaf and leaf.requires_grad and torch.equal(leaf.detach(), value)
        assert leaf.grad.data_ptr() == flat.view(grad, name).data_ptr()
    a, b = flat.leaves["a"], flat.leaves["b"]
    (2.0 * a.sum() + (b * b).sum()).backward()
    (a * 3.0).sum().backward()  # a second use of the same leaf adds in place
    assert torch.equal(flat.view(grad, "a"), torch.full((3, 4), 5.0))
    torch.testing.assert_close(flat.view(grad, "b"), 2.0 * params["b"])
    assert torch.equal(flat.view(grad, "c"), torch.zeros(2, 2, 2))
    with torch.no_grad():
        flat.master.add_(1.0)  # an optimizer writing the master moves every leaf
    torch.testing.assert_close(a.detach(), params["a"] + 1.0)


def test_lookup_one_hot_product_is_exact_and_scatters_gradients():
    from pbg_b200.preflop import lookup

    gen = torch.Generator().manual_seed(1)
    table = torch.randn(9, 16, generator=gen)
    index = torch.randint(0, 9, (7, 11), generator=gen)
    plain = lookup(table, index)
    assert torch.equal(plain, table[index])
    leaf = table.clone().requires_grad_()
    rows = lookup(leaf, index)
    assert torch.equal(rows.detach(), table[index])
    weight = torch.randn(rows.shape, generator=gen)
    (rows * weight).sum().backward()
    want = torch.zeros_like(table).index_add_(0, index.reshape(-1), weight.reshape(-1, 16))
    torch.testing.assert_close(leaf.grad, want, rtol=1e-6, atol=1e-6)


def test_training_pad_matches_inference_pad():
    from pbg_b200.preflop import _padded

    gen = torch.Generator().manual_seed(2)
    x = torch.randn(6, 50, generator=gen)
    eval_rows = _padded(x, 64)
    leaf = x.clone().requires_grad_()
    train_rows = _padded(leaf, 64)
    assert train_rows.dtype == torch.bfloat16 and train_rows.shape == (6, 64)
    assert torch.equal(train_rows.detach(), eval_rows)
    weight = torch.randn(6, 64, generator=gen)
    (train_rows.float() * weight).sum().backward()
    torch.testing.assert_close(leaf.grad, weight[:, :50].to(torch.bfloat16).float())


def _preflop_model():
    import model_params
    from pbg_b200.preflop import PreflopConfig, PreflopModel, parameter_shapes

    cfg = PreflopConfig(**model_params.CONFIG)
    params = {n: torch.from_numpy(model_params.parameter(n, s)) for n, s in parameter_shapes(cfg, 4).items()}
    return PreflopModel(cfg, 4, params, "cpu"), params


def test_bound_parameters_drive_the_fused_maps():
    from pbg_b200.model_train import FlatParameters, q_scale_of

    model, params = _preflop_model()
    flat = FlatParameters(model.p, "cpu")
    model.bind_parameters(flat.leaves)
    layer = model.layers[0]
    # FamilyFFN's common and static maps are one map over [x, s]: its source concatenates the leaves
    w, b = layer["ffn_in"].source()
    want = torch.cat((params["layer_ffns.0.common.weight"], params["layer_ffns.0.static.pre.weight"]), 1)
    assert torch.equal(w.detach(), want) and b is flat.leaves["layer_ffns.0.common.bias"]
    # incidence query / identical / own as one map over [n | oe | own]
    w, _ = layer["inc_in"].source()
    assert w.shape == (128, 3 * 128) and w.requires_grad
    # a parameter update reaches the bf16 operand of its map and the head scales after sync_weights
    with torch.no_grad():
        flat.leaves["attentions.0.w_qkv.weight"].mul_(2.0)
        flat.leaves["attentions.0.theta"].add_(0.25)
    model.sync_weights()
    qkv = layer["w_qkv"]
    torch.testing.assert_close(qkv.weight[: qkv.n, : qkv.k].float(),
                               (2.0 * params["attentions.0.w_qkv.weight"]).to(torch.bfloat16).float())
    theta = params["attentions.0.theta"] + 0.25
    torch.testing.assert_close(layer["q_scale"], 1.0 / ((torch.nn.functional.softplus(theta) + 0.5) * math.sqrt(32)))
    torch.testing.assert_close(q_scale_of(theta), layer["q_scale"])
    assert not model.binding.training
    model.train()
    assert model.binding.training and all(m.binding is model.binding for m in model._maps)
    model.train(False)
    assert not model.binding.training


def test_model_params_probe_is_seeded_by_name():
    import model_params

    a = model_params.probe("x.weight", (3, 4))
    assert a.shape == (model_params.SKETCH_PROBES, 12)
    assert np.array_equal(a, model_params.probe("x.weight", (3, 4)))
    assert not np.array_equal(a, model_params.probe("y.weight", (3, 4)))
