"""The preflop network's class geometry (sizes, orbit-averaged card incidence, overlap scalars)
restated in pbg_b200.preflop against the reference's own buffers (preflop.py:234-253)."""

import numpy as np
import torch


def test_class_geometry_matches_reference_buffers(gold):
    from pbg_b200.preflop import class_geometry

    d = gold("preflop_model")
    sizes, orbit, overlap = class_geometry(4)
    np.testing.assert_array_equal(sizes.numpy(), d["class_sizes"])
    np.testing.assert_allclose(orbit.numpy(), d["class_card_geometry"], rtol=0, atol=1e-7)
    np.testing.assert_allclose(overlap.numpy(), d["class_overlap_scalars"], rtol=1e-6, atol=1e-7)


def test_parameter_shapes_match_reference_modules(gold):
    import os
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import model_params
    from pbg_b200.preflop import PreflopConfig, parameter_shapes

    d = gold("preflop_model")
    reference = {}
    for item in d["param_spec"]:
        name, dims = str(item).split(":")
        reference[name] = tuple(int(x) for x in dims.split(","))
    assert parameter_shapes(PreflopConfig(**model_params.CONFIG), model_params.RANKS) == reference
