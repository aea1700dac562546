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

`compile_package` compiles the packages with the library's C shims (`C_SHIMS`): the package calls
`aoti_torch_cuda_fold(...)` and its siblings directly, instead of a boxed call through AOTInductor's
proxy executor. The process that runs such a package must have loaded LIB with RTLD_GLOBAL (what
`load()` does; a C++ host dlopens it with RTLD_GLOBAL) so the package resolves those symbols.
It also runs `inductor_pass` (a float16/bfloat16 region's widening input cast and narrowing
output cast folded into the kernel, which reads the 16-bit storage itself).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libneptune_b200_torch.so")
SOURCE = os.path.join(HERE, "csrc", "torch_ops.cpp")
EXPORTS = os.path.join(HERE, "csrc", "torch_ops.map")  # only the C shims are exported
BUILD_DIR = os.path.join(HERE, "csrc", "_build", "torch_ops")

_LOADED = False


def build(verbose: bool = False) -> str:
    """Compile csrc/torch_ops.cpp against the installed torch into LIB (no GPU needed)."""
    from torch.utils import cpp_extension

    os.makedirs(BUILD_DIR, exist_ok=True)
    cpp_extension.load(name="neptune_b200_torch", sources=[SOURCE], extra_cflags=["-O2", "-std=c++17"],
                       extra_ldflags=["-ldl", f"-Wl,--version-script={EXPORTS}"], with_cuda=True,
                       build_directory=BUILD_DIR, is_python_module=False, verbose=verbose)
    shutil.copy2(os.path.join(BUILD_DIR, "neptune_b200_torch.so"), LIB)
    import ctypes

    # the copy cpp_extension.load just opened, made global: the C shims, for packages loaded here
    ctypes.CDLL(os.path.join(BUILD_DIR, "neptune_b200_torch.so"), mode=ctypes.RTLD_GLOBAL)
    global _LOADED
    _LOADED = True  # cpp_extension.load registered the ops in this process
    return LIB


def load() -> None:
    """Register the nb200 ops in this process (fails loudly when the library is not built). The
    library is opened with RTLD_GLOBAL so that packages compiled with its C shims (`c_shims()`)
    resolve them when they are loaded."""
    global _LOADED
    if _LOADED:
        return
    import ctypes

    import torch

    if not os.path.exists(LIB):
        from neptune_opt_b200._lib import BackendUnavailable

        raise BackendUnavailable(f"{LIB} is not built; run neptune_opt_b200.aot.build()")
    ctypes.CDLL(LIB, mode=ctypes.RTLD_GLOBAL)
    torch.ops.load_library(LIB)
    _LOADED = True


# The C entry points of csrc/torch_ops.cpp, in AOTInductor's C-shim conventions.
C_SHIMS = {
    "fold": "AOTITorchError aoti_torch_cuda_fold(AtenTensorHandle x, int64_t skeleton, const double* params, "
            "int64_t params_len_, int32_t keepdim, int64_t plan, int64_t block, int64_t num_warps, "
            "AtenTensorHandle* ret0)",
    "softmax": "AOTITorchError aoti_torch_cuda_softmax(AtenTensorHandle x, int64_t mode, AtenTensorHandle* ret0, "
               "AtenTensorHandle* ret1)",
    "l2_normalize": "AOTITorchError aoti_torch_cuda_l2_normalize(AtenTensorHandle x, AtenTensorHandle* ret0, "
                    "AtenTensorHandle* ret1)",
    "rms_norm": "AOTITorchError aoti_torch_cuda_rms_norm(AtenTensorHandle x, AtenTensorHandle gamma, double eps, "
                "AtenTensorHandle* ret0)",
    "segment_pool": "AOTITorchError aoti_torch_cuda_segment_pool(AtenTensorHandle data, AtenTensorHandle segments, "
                    "int32_t offsets, int64_t reduce, double* initial, int32_t unsafe, AtenTensorHandle* ret0)",
    "attention": "AOTITorchError aoti_torch_cuda_attention(AtenTensorHandle q, AtenTensorHandle k, AtenTensorHandle v, "
                 "int32_t causal, double scale, AtenTensorHandle* ret0, AtenTensorHandle* ret1)",
}


def c_shims() -> dict:
    """`aot_inductor.custom_ops_to_c_shims` for the nb200 ops: a package compiled with it calls the
    library's C entry points directly instead of through the proxy executor's boxed call."""
    import torch

    load()
    return {getattr(torch.ops.nb200, name).default: [decl] for name, decl in C_SHIMS.items()}


def enable_c_shims() -> None:
    """Make every later AOTInductor compilation in this process (the reference's compile_best
    included) call the nb200 ops through their C shims."""
    import torch._inductor.config as cfg

    cfg.aot_inductor.custom_ops_to_c_shims = {**cfg.aot_inductor.custom_ops_to_c_shims, **c_shims()}


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


def compile_package(exported, package_path: str | None = None, *, shims: bool = True,
                    fuse_casts: bool = True) -> str:
    """torch._inductor.aoti_compile_and_package with a host compiler that builds OpenMP code,
    (shims=True) the nb200 ops called through their C shims and (fuse_casts=True) the regions'
    widening input casts folded into their kernels (`inductor_pass`)."""
    import torch
    import torch._inductor.config as cfg

    patch = {"cpp.cxx": (None, host_compiler())}
    if shims:
        patch["aot_inductor.custom_ops_to_c_shims"] = {**cfg.aot_inductor.custom_ops_to_c_shims, **c_shims()}
    if fuse_casts and type(cfg.post_grad_custom_post_pass).__name__ != "CastFusion":
        from neptune_opt_b200 import inductor_pass

        patch["post_grad_custom_post_pass"] = inductor_pass.make_pass(cfg.post_grad_custom_post_pass)
    with cfg.patch(patch):
        return torch._inductor.aoti_compile_and_package(exported, package_path=package_path)
