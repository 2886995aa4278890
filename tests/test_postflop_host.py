"""Host-side parts of the postflop family: parameter names/shapes and the compact row map.

The compact map (incidence.py:111-216) is checked against a loop restatement of its contract:
compatible rows in increasing full-row order, padding reads as zero on gather, omitted rows take the
fill value on scatter.  The parameter table is checked against the reference modules' own
``named_parameters`` as recorded in tests/golden/postflop_model.npz.
"""

import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def test_parameter_shapes_match_reference_modules(gold):
    import model_params
    from pbg_b200.postflop import parameter_shapes
    from pbg_b200.preflop import PreflopConfig

    d = gold("postflop_model")
    spec = {}
    for item in d["param_spec"]:
        name, dims = str(item).split(":")
        spec[name] = tuple(int(x) for x in dims.split(","))
    assert parameter_shapes(PreflopConfig(**model_params.POSTFLOP_CONFIG), model_params.RANKS) == spec


def _loop_map(compat, q):
    batch, full = compat.shape
    c2f = np.zeros((batch, q), dtype=np.int64)
    f2c = np.full((batch, full), -1, dtype=np.int64)
    valid = np.zeros((batch, q), dtype=bool)
    for b in range(batch):
        rows = [h for h in range(full) if compat[b, h]]
        for i, h in enumerate(rows):
            c2f[b, i], f2c[b, h], valid[b, i] = h, i, True
    return c2f, f2c, valid


@pytest.mark.parametrize("seed,batch,full,density,slack", [(0, 3, 120, 0.7, 0), (1, 5, 31, 0.3, 4),
                                                            (2, 2, 16, 0.0, 2), (3, 4, 45, 1.0, 0)])
def test_compact_map_gather_scatter(seed, batch, full, density, slack):
    from pbg_b200.postflop import build_compact_map, compact_gather, compact_scatter

    g = torch.Generator().manual_seed(seed)
    compat = torch.rand((batch, full), generator=g) < density
    q = int(compat.sum(1).max()) + slack
    mapping = build_compact_map(compat, q)
    c2f, f2c, valid = _loop_map(compat.numpy(), q)
    assert np.array_equal(mapping.full_to_compact.numpy(), f2c)
    assert np.array_equal(mapping.valid.numpy(), valid)
    assert np.array_equal(mapping.compact_to_full.numpy()[valid], c2f[valid])
    values = torch.randn((batch, 3, full, 2), generator=g)
    gathered = compact_gather(values, mapping, dim=2)
    want = np.zeros((batch, 3, q, 2), dtype=np.float32)
    for b in range(batch):
        for i in range(q):
            if valid[b, i]:
                want[b, :, i] = values[b, :, c2f[b, i]].numpy()
    assert np.array_equal(gathered.numpy(), want)
    back = compact_scatter(gathered, mapping, dim=2, fill_value=7.0)
    expect = torch.where(compat[:, None, :, None], values, torch.full_like(values, 7.0))
    assert torch.equal(back, expect)


def test_compact_map_rejects_bad_inputs():
    from pbg_b200.postflop import build_compact_map

    with pytest.raises(TypeError):
        build_compact_map(torch.ones((2, 4)))
    with pytest.raises(ValueError):
        build_compact_map(torch.ones((2, 4), dtype=torch.bool), 5)
    with pytest.raises(ValueError, match="omits compatible rows"):
        build_compact_map(torch.ones((2, 4), dtype=torch.bool), 3)


def test_queued_parameter_shapes_match_reference_module(gold):
    import model_params
    from pbg_b200.preflop import PreflopConfig
    from pbg_b200.queued_model import parameter_shapes

    d = gold("queued_model")
    spec = {}
    for item in d["param_spec"]:
        name, dims = str(item).split(":")
        spec[name] = tuple(int(x) for x in dims.split(","))
    history, players = (int(x) for x in d["config"])
    cfg = PreflopConfig(**dict(model_params.CONFIG, max_players=players, max_history_tokens=history))
    assert parameter_shapes(cfg, model_params.RANKS, branching_heads=True) == spec
