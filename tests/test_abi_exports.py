"""The C-ABI library loads and exports every symbol include/pbgb200.h declares.

Runs without a GPU: nothing is launched.
"""

import ctypes
import os
import re

from conftest import ROOT


def _declared():
    text = open(os.path.join(ROOT, "include", "pbgb200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pbg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    from pbg_b200 import _native

    lib = _native.lib()
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding declares a signature for every exported entry point
    assert set(names) <= set(_native.SIGNATURES), set(names) - set(_native.SIGNATURES)
    assert lib.pbg_abi_version() == 1


def test_errors_are_reported_without_a_device():
    from pbg_b200 import _native

    lib = _native.lib()
    rc = lib.pbg_rng_keys(0, 0, 0, 1, None, None, None, None, None, None, None, None)
    assert rc == -1
    assert b"purpose" in lib.pbg_last_error()
    g = _native.Geometry(7, 16, 13)
    assert lib.pbg_combo_class(g, None, None) == -1
    assert b"players" in lib.pbg_last_error()


def test_python_layer_refuses_cpu_tensors():
    import pytest
    import torch
    from pbg_b200 import rng
    from pbg_b200._native import NativeError

    with pytest.raises(NativeError):
        rng.logical_uniform(torch.zeros(4, dtype=torch.int64))
