"""The compact postflop policy/value network on this build's kernels against the reference module itself.

tests/golden/postflop_model*.npz hold the reference PostflopEncoder's fp32 outputs (run on CPU by
tests/golden/make_golden.py) at three configurations (d128 / 2 layers at 4 ranks; the cfg2 network
and the reference's default network at 13 ranks): three seats with one folded (so the folded-seat summary and the folder
context are live), flop and turn boards, the board-compatible compact rows, random evaluator-summary
fields and fold-line features, weights drawn by tests/golden/model_params.py from the parameter
names.  This build runs the same weights in bf16 on the tensor cores (fp32 accumulation, fp32
residual stream).  Tolerance: the bf16 bar, rtol and atol 2e-2.
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def _params(d):
    import model_params

    params = {}
    for item in d["param_spec"]:
        name, dims = str(item).split(":")
        params[name] = torch.from_numpy(model_params.parameter(name, tuple(int(x) for x in dims.split(","))))
    return params


def _model(params, d=None):
    """The network of a fixture: its recorded configuration and rank count (the small default
    fixture predates the record and uses model_params.POSTFLOP_CONFIG at model_params.RANKS)."""

    import json

    import model_params
    from pbg_b200.postflop import PostflopModel
    from pbg_b200.preflop import PreflopConfig

    if d is not None and "config_json" in d:
        return PostflopModel(PreflopConfig(**json.loads(str(d["config_json"]))), int(d["ranks"]), params, DEV)
    return PostflopModel(PreflopConfig(**model_params.POSTFLOP_CONFIG), model_params.RANKS, params, DEV)


def _inputs(d):
    from pbg_b200.postflop import PostflopMasks

    pub = {k[4:]: torch.from_numpy(d[k]).to(DEV) for k in d if k.startswith("pub_")}
    pub["history"] = {k[5:]: torch.from_numpy(d[k]).to(DEV) for k in d if k.startswith("hist_")}
    summary = {k[8:]: torch.from_numpy(d[k]).to(DEV) for k in d if k.startswith("summary_")}
    masks = PostflopMasks(compatibility=torch.from_numpy(d["compatibility"]).to(DEV), evaluator_summary=summary,
                          fold_line_features=torch.from_numpy(d["fold_line_features"]).to(DEV),
                          compact_size=int(d["compact_size"]))
    return pub, torch.from_numpy(d["combo_ranges"]).to(DEV), masks


def _worst(raw, value, d):
    diffs = {k: float((raw[k].cpu() - torch.from_numpy(d["raw_" + k])).abs().max()) for k in raw}
    diffs["value"] = float((value.cpu() - torch.from_numpy(d["value"])).abs().max())
    return diffs


@pytest.mark.parametrize("fixture", ["postflop_model", "postflop_model_r13", "postflop_model_default"])
def test_postflop_forward_matches_reference_module(gold, fixture):
    """d128 / 2 layers at 4 ranks; the cfg2 network (d128, 2 layers, 4 heads, M = 2, FFN 512) and the
    reference's default network (d256, 8 heads, 6 layers) at 13 ranks, whose 3 x ~1,176 compact rows per
    decision run the attention kernel's multi-tile and tail paths."""

    d = gold(fixture)
    model = _model(_params(d), d)
    pub, ranges, masks = _inputs(d)
    raw, value = model.forward(pub, ranges, None, masks)
    torch.cuda.synchronize()
    from pbg_b200.postflop import input_errors

    assert input_errors(DEV) == []
    print("\nmax |b200 - reference|:", _worst(raw, value, d))
    assert set(raw) == {k[4:] for k in d if k.startswith("raw_")}
    for k in raw:
        torch.testing.assert_close(raw[k].cpu(), torch.from_numpy(d["raw_" + k]), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(value.cpu(), torch.from_numpy(d["value"]), rtol=2e-2, atol=2e-2)


def test_postflop_selected_private_row_is_the_full_row(gold):
    # postflop.py:747-752: the learner's one selected hand equals that hand's row of the full output
    d = gold("postflop_model")
    model = _model(_params(d))
    pub, ranges, masks = _inputs(d)
    compat = masks.compatibility
    selected = compat.float().argmax(1) + 1  # a board-compatible hand of each decision
    selected = torch.where(compat.gather(1, selected[:, None]).squeeze(1), selected, compat.float().argmax(1))
    raw, value = model.forward(pub, ranges, None, masks, selected_private=selected)
    full, full_value = model.forward(pub, ranges, None, masks)
    rows = torch.arange(selected.shape[0], device=DEV)
    for k in raw:
        torch.testing.assert_close(raw[k][:, 0], full[k][rows, selected], rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(value[:, 0], full_value[rows, selected], rtol=1e-3, atol=1e-3)


def test_postflop_forward_detects_a_changed_weight(gold):
    # the tolerance above is far below what one perturbed postflop-only weight does to the outputs
    d = gold("postflop_model")
    params = dict(_params(d))
    params["folder_context.w2.weight"] = params["folder_context.w2.weight"] * 3.0
    pub, ranges, masks = _inputs(d)
    raw, value = _model(params).forward(pub, ranges, None, masks)
    assert max(_worst(raw, value, d).values()) > 0.05


def test_postflop_input_check_records_a_folded_actor(gold):
    # postflop.py:409-412: the actor seat must be present; seat 2 is folded in every decision of the
    # fixture.  The check is recorded on the device (every index stays in range) and raised on the host.
    from pbg_b200.postflop import input_errors, raise_input_errors

    d = gold("postflop_model")
    model = _model(_params(d))
    pub, ranges, masks = _inputs(d)
    input_errors(DEV)
    model.forward(pub, ranges, torch.full((ranges.shape[0],), 2, dtype=torch.long, device=DEV), masks)
    with pytest.raises(ValueError, match="the actor seat must be present"):
        raise_input_errors(DEV)
    assert input_errors(DEV) == []
