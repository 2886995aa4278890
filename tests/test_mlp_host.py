"""Host logic of the cfg1 MLP learner step that runs without a GPU: the chunked weight gradient
(pbg_b200.mlp._weight_gradient) equals dy^T x for row counts with and without a remainder, and the
flat parameter layout covers every tensor once."""

import math

import pytest
import torch


@pytest.mark.parametrize("S", [1, 511, 512, 1024, 1537, 4096 + 300])
def test_chunked_weight_gradient_equals_the_plain_product(S):
    from pbg_b200.mlp import _weight_gradient

    g = torch.Generator().manual_seed(S)
    dy = torch.randn(S, 17, generator=g, dtype=torch.float64)
    x = torch.randn(S, 9, generator=g, dtype=torch.float64)
    out = torch.empty(17, 9, dtype=torch.float64)
    _weight_gradient(dy, x, out)
    torch.testing.assert_close(out, dy.t() @ x, rtol=1e-12, atol=1e-12)


def test_flat_parameter_layout():
    from pbg_b200.mlp import PreflopMLP
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    model = PreflopMLP(geometry, device="cpu", seed=3)
    assert model.out == geometry.private_classes * (4 + 3 * 2) + geometry.private_classes
    assert model.numel == sum(math.prod(shape) for _, shape in model.shapes) == model.master.numel()
    views = model.views(model.master)
    assert sum(v.numel() for v in views.values()) == model.numel
    assert views["w1"].shape == (256, geometry.preflop_model_input_width)
    bound = 1.0 / math.sqrt(geometry.preflop_model_input_width)
    assert float(views["w1"].abs().max()) <= bound
