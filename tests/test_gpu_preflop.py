"""The preflop policy/value network on this build's kernels against the reference module itself.

tests/golden/preflop_model*.npz hold the reference PreflopEncoder's fp32 outputs at three
configurations (d128 / 2 layers at 4 ranks; the cfg2 network and the default network at 13 ranks) (run on CPU by
tests/golden/make_golden.py) for seeded public batches and ranges, with weights drawn by
tests/golden/model_params.py from the parameter names; this build runs the same weights in bf16
on the tensor cores (fp32 accumulation, fp32 residual stream).  Tolerance: the bf16 bar, rtol and
atol 2e-2 (observed worst case about 8e-3 on the type logits).
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def _model(d):
    """The network of a fixture: its recorded configuration and rank count (the small default fixture
    predates the record and uses model_params.CONFIG at model_params.RANKS)."""

    import json

    import model_params
    from pbg_b200.preflop import PreflopConfig, PreflopModel

    params = {}
    for item in d["param_spec"]:
        name, dims = str(item).split(":")
        shape = tuple(int(x) for x in dims.split(","))
        params[name] = torch.from_numpy(model_params.parameter(name, shape))
    if "config_json" in d:
        cfg, ranks = PreflopConfig(**json.loads(str(d["config_json"]))), int(d["ranks"])
    else:
        cfg, ranks = PreflopConfig(**model_params.CONFIG), model_params.RANKS
    return PreflopModel(cfg, ranks, params, DEV), params


def _pub(d):
    pub = {k[4:]: torch.from_numpy(d[k]).to(DEV) for k in d if k.startswith("pub_")}
    pub["history"] = {k[5:]: torch.from_numpy(d[k]).to(DEV) for k in d if k.startswith("hist_")}
    return pub


@pytest.mark.parametrize("fixture", ["preflop_model", "preflop_model_r13", "preflop_model_default"])
def test_preflop_forward_matches_reference_module(gold, fixture):
    """d128 / 2 layers at 4 ranks; the cfg2 network and the reference's default network (d256, 8 heads,
    6 layers) at 13 ranks (169 class rows per seat, 2 x 169 + public + history + anchor tokens)."""

    d = gold(fixture)
    model, _ = _model(d)
    raw, value = model.forward(_pub(d), torch.from_numpy(d["class_ranges"]).to(DEV),
                               torch.from_numpy(d["class_mask"]).to(DEV))
    torch.cuda.synchronize()
    diffs = {k: float((raw[k].cpu() - torch.from_numpy(d["raw_" + k])).abs().max()) for k in raw}
    diffs["value"] = float((value.cpu() - torch.from_numpy(d["value"])).abs().max())
    print("\nmax |b200 - reference|:", diffs)
    for k in raw:
        torch.testing.assert_close(raw[k].cpu(), torch.from_numpy(d["raw_" + k]), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(value.cpu(), torch.from_numpy(d["value"]), rtol=2e-2, atol=2e-2)


def test_preflop_forward_detects_a_changed_weight(gold):
    # the tolerance above is far below what one perturbed weight matrix does to the outputs
    import model_params
    from pbg_b200.preflop import PreflopConfig, PreflopModel

    d = gold("preflop_model")
    _, params = _model(d)
    params = dict(params)
    params["layer_ffns.1.output.weight"] = params["layer_ffns.1.output.weight"] * 1.5
    model = PreflopModel(PreflopConfig(**model_params.CONFIG), model_params.RANKS, params, DEV)
    raw, value = model.forward(_pub(d), torch.from_numpy(d["class_ranges"]).to(DEV),
                               torch.from_numpy(d["class_mask"]).to(DEV))
    worst = max(float((raw[k].cpu() - torch.from_numpy(d["raw_" + k])).abs().max()) for k in raw)
    assert worst > 0.1
