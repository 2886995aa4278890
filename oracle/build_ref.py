"""Compile the reference's own native operators into oracle/_ref (test infrastructure only).

    python oracle/build_ref.py [--reference <pbg checkout>] [--force]

The checkout is the ``--reference`` argument, else ``$PBG_REFERENCE``, else a
directory named ``reference`` beside this repository; with none of them
present nothing is built.

The reference's native operators are single CUDA source files, each a torch
extension with one entry point: pbg/core/csrc/layered_targets.cu
(``run_layers``), alias_table.cu (``build_alias_table``) and
branching_metadata.cu (``decision_log_mass``).  This recipe compiles each file
where it lies in the pbg checkout with the reference's own device flags
(pbg/core/cuda_layer.py:19-25, cuda_alias.py, cuda_branching.py: -O3
--fmad=false) for sm_100a, linking the torch libraries of this interpreter,
into ``oracle/_ref/<module><EXT_SUFFIX>``.  Nothing is
copied into this repository.  The GPU tests import the module (when it was
built) to check the CUDA library against the reference's kernel itself; the
product never loads it.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
MODULES = {
    "ref_layered_targets": os.path.join("pbg", "core", "csrc", "layered_targets.cu"),
    "ref_alias_table": os.path.join("pbg", "core", "csrc", "alias_table.cu"),
    "ref_branching_metadata": os.path.join("pbg", "core", "csrc", "branching_metadata.cu"),
}
MODULE = "ref_layered_targets"
DEFAULT_REFERENCE = os.environ.get(
    "PBG_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def target(module: str = MODULE) -> str:
    return os.path.join(OUT, module + sysconfig.get_config_var("EXT_SUFFIX"))


def build(reference: str = DEFAULT_REFERENCE, force: bool = False) -> str | None:
    """Build every reference operator (in parallel); None when the pbg checkout is absent."""

    if not os.path.exists(os.path.join(reference, MODULES[MODULE])):
        return None
    jobs = []
    for module in MODULES:
        cmd = _command(reference, module, force)
        if cmd is not None:
            jobs.append(subprocess.Popen(cmd))
    for job in jobs:
        if job.wait() != 0:
            raise RuntimeError("building a reference operator failed")
    return target()


def _command(reference: str, module: str, force: bool) -> list[str] | None:
    src = os.path.join(reference, MODULES[module])
    out = target(module)
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
        return None
    import torch
    from torch.utils import cpp_extension

    os.makedirs(OUT, exist_ok=True)
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    includes = cpp_extension.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [os.path.join(cuda, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--fmad=false",
           "-std=c++17", "-shared", "-Xcompiler", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-DTORCH_EXTENSION_NAME={module}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "--expt-relaxed-constexpr", "-o", out, src]
    for inc in includes:
        cmd += ["-I", inc]
    for lib in libs:
        cmd += ["-L", lib, f"-Xlinker=-rpath,{lib}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    return cmd


def load(module: str = MODULE):
    """Import a built module, or None when it was not built."""

    path = target(module)
    if not os.path.exists(path):
        return None
    import importlib.util

    import torch  # noqa: F401  (the module links libtorch)

    spec = importlib.util.spec_from_file_location(module, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    result = build(a.reference, a.force)
    print(result if result else f"no pbg checkout at {a.reference}: nothing built")
    sys.exit(0)
