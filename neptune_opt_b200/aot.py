"""The region ops registered from C++ (`torch.ops.nb200.*`), for AOTInductor packages.

The reference routes its regions into AOTInductor as Triton ops that Inductor copies into the
package (neptune_codegen/torch_op.py:16-114, packaged by neptune_opt/ab.py:145-172). Here the
kernels are hand-written CUDA behind a C ABI, so the package instead calls the ops by name through
the dispatcher; `libneptune_b200_torch.so` (csrc/torch_ops.cpp) registers them with C++ kernels,
so a compiled package runs them with no Python op layer at all -- the library only has to be
loaded into the process that runs the package (`load()`, or `torch.ops.load_library(LIB)`).

    import neptune_opt_b200.aot as A
    A.load()
    y = A.fold(x, "logsumexp")                       # torch.ops.nb200.fold(x, 0, [...], False, 0, 0)
    ep = torch.export.export(model, args)            # model calls torch.ops.nb200.*
    pkg = A.compile_package(ep, "regions.pt2")       # aoti_compile_and_package, see below
    runner = torch._inductor.aoti_load_package(pkg)  # in any process that loaded LIB

The ops take their skeleton and parameters as arguments (one op per region kind) instead of
baking them into the op name as the Python layer's per-key ops do: a C++ library registers its
ops once at load, before any graph names a parameter set.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libneptune_b200_torch.so")
SOURCE = os.path.join(HERE, "csrc", "torch_ops.cpp")
BUILD_DIR = os.path.join(HERE, "csrc", "_build", "torch_ops")

_LOADED = False


def build(verbose: bool = False) -> str:
    """Compile csrc/torch_ops.cpp against the installed torch into LIB (no GPU needed)."""
    from torch.utils import cpp_extension

    os.makedirs(BUILD_DIR, exist_ok=True)
    cpp_extension.load(name="neptune_b200_torch", sources=[SOURCE], extra_cflags=["-O2", "-std=c++17"],
                       extra_ldflags=["-ldl"], with_cuda=True, build_directory=BUILD_DIR,
                       is_python_module=False, verbose=verbose)
    shutil.copy2(os.path.join(BUILD_DIR, "neptune_b200_torch.so"), LIB)
    global _LOADED
    _LOADED = True  # cpp_extension.load registered the ops in this process
    return LIB


def load() -> None:
    """Register the nb200 ops in this process (fails loudly when the library is not built)."""
    global _LOADED
    if _LOADED:
        return
    import torch

    if not os.path.exists(LIB):
        from neptune_opt_b200._lib import BackendUnavailable

        raise BackendUnavailable(f"{LIB} is not built; run neptune_opt_b200.aot.build()")
    torch.ops.load_library(LIB)
    _LOADED = True


def fold_params(name: str, params: dict | None = None) -> list:
    """[tiny, alpha, T, beta, N, eps] for skeleton `name`, with its defaults and domain checks."""
    from neptune_opt_b200.skeletons import checked_params, param_defaults

    v = checked_params(name, {**param_defaults(name), **(params or {})})
    return [float(v.get("tiny", 0.0)), float(v.get("alpha", 0.0)), float(v.get("T", 1.0)),
            float(v.get("beta", 1.0)), float(v.get("N", 1.0)), float(v.get("eps", 1.0))]


def fold(x, name: str, params: dict | None = None, *, keepdim: bool = False, plan: str = "serial",
         block: int | None = None):
    """torch.ops.nb200.fold for skeleton `name` (serial or split plan)."""
    import torch

    from neptune_opt_b200.skeletons import SKELETONS
    from neptune_opt_b200.template import validate_plan

    validate_plan(plan)
    load()
    return torch.ops.nb200.fold(x, SKELETONS[name].id, fold_params(name, params), keepdim,
                                0 if plan == "serial" else 1, int(block or 0))


def _cxx_builds_openmp(cxx: str) -> bool:
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.cpp")
        with open(src, "w") as f:
            f.write("#include <omp.h>\nint main() { return omp_get_max_threads() > 0 ? 0 : 1; }\n")
        try:
            return subprocess.run([cxx, "-fopenmp", src, "-o", os.path.join(d, "t")], capture_output=True,
                                  timeout=120).returncode == 0
        except (OSError, subprocess.TimeoutExpired):
            return False


def host_compiler() -> str:
    """The C++ compiler AOTInductor should use: its configured one when that builds OpenMP code
    (the generated wrapper is compiled with -fopenmp), else the first of g++ / c++ on the system
    that does."""
    import torch._inductor.config as cfg

    configured = cfg.cpp.cxx[-1] if isinstance(cfg.cpp.cxx, tuple) else cfg.cpp.cxx
    for cxx in (configured, "/usr/bin/g++", "/usr/bin/c++", "g++"):
        if cxx and _cxx_builds_openmp(cxx):
            return cxx
    return configured


def compile_package(exported, package_path: str | None = None) -> str:
    """torch._inductor.aoti_compile_and_package with a host compiler that builds OpenMP code."""
    import torch
    import torch._inductor.config as cfg

    with cfg.patch({"cpp.cxx": (None, host_compiler())}):
        return torch._inductor.aoti_compile_and_package(exported, package_path=package_path)
