"""Graphs rewritten by the reference's own front end, run on the GPU through this backend.

The fixtures (tests/golden/rewrite_*.pt2, made by tests/golden/make_rewrites.py) are what the
reference's unchanged `neptune_opt.apply` produced with this backend bound in. Here, without the
reference:
1. each rewritten program runs eagerly on the GPU and matches the CPU oracle at the parity bars;
2. each is compiled by AOTInductor -- the packaging step of the reference's `compile_best`
   (neptune_opt/ab.py:145-172) -- and the package, run in a fresh process that loads only the C++
   op library (no neptune_opt_b200 Python, no per-key op registrations), reproduces the eager
   results bit for bit.
3. When the reference itself is installed under baseline/_ref, its whole surface runs on the GPU
   with this backend: `apply(ep, verify_with=...)` reports a verified fusion, and `compile_best`
   compiles, verifies and times the fused package (neptune_opt/ab.py:270-530).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import assert_close_dtype, assert_rms_close, cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
ROOT = os.path.dirname(HERE)
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

with open(os.path.join(GOLDEN, "rewrites.json")) as _f:
    CASES = sorted(json.load(_f)["cases"])


def _check_against_oracle(name, args, got, oracle_mod):
    import torch

    x = args[0].float().cpu().numpy()
    out = got.float().cpu().numpy()
    if name in ("logsumexp_f32", "shifted_exp_sum_f32"):
        ref = oracle_mod.fold("logsumexp", x, {"tiny": 0.0})
        if name == "shifted_exp_sum_f32":
            ref = ref * np.float32(0.5)  # the graph's own multiply after the region (exact)
        assert_close_dtype(out, ref, "float32", rtol32=1e-5)
    elif name == "row_l2_f32":
        assert_close_dtype(out, oracle_mod.fold("stable_l2", x, {}), "float32", rtol32=1e-5)
    elif name == "logsumexp_split_bf16":
        # the reference lowers the bf16 region to fp32 around the op: fp32 fold, then a bf16 cast
        ref = oracle_mod.fold("logsumexp", x, {"tiny": 0.0}, block=1024)
        assert_close_dtype(out, ref, "bfloat16")
    elif name == "rms_norm_bf16":
        gamma = args[1].float().cpu().numpy()
        assert_rms_close(out, oracle_mod.rms_norm(x, gamma, 1e-6, "bfloat16"), "bfloat16")
    elif name == "segment_mean_f16":
        lengths = args[1].cpu().numpy()
        spans, status = oracle_mod.segment_spans(lengths, False, False, x.shape[0])
        want = oracle_mod.segment_pool(x, spans, "mean", None, "float16")
        assert status == 0 and np.array_equal(out, want)
    else:
        raise AssertionError(f"no oracle check for {name}")
    assert got.dtype == args[0].dtype and got.device.type == "cuda"
    del torch


@pytest.mark.parametrize("name", CASES)
def test_rewritten_program_runs_and_matches_the_oracle(name, oracle_mod):
    import torch

    import neptune_opt_b200 as NB
    import rewrite_models
    from make_rewrites import load_case

    ep, _case = load_case(name)
    args = rewrite_models.CASES[name][1]("cuda")
    before = NB.launch_count()
    got = ep.module()(*args)
    torch.cuda.synchronize()
    assert NB.launch_count() > before, "the rewritten graph did not launch this library's kernels"
    _check_against_oracle(name, args, got, oracle_mod)


def test_rewritten_programs_package_and_run_without_python_ops(tmp_path, oracle_mod):
    import torch

    import neptune_opt_b200.aot as A
    import rewrite_models
    from make_rewrites import load_case

    from neptune_opt_b200.inductor_pass import fuse_casts

    jobs = []
    for name in CASES:
        ep, _case = load_case(name)
        args = rewrite_models.CASES[name][1]("cuda")
        # the package runs the graph with its 16-bit regions' casts folded into the kernels
        # (compile_package's cast-fusion pass): run the same graph eagerly
        eager_gm = ep.run_decompositions().module()
        fused = fuse_casts(eager_gm.graph)
        assert fused == (1 if name == "logsumexp_split_bf16" else 0), (name, fused)
        eager_gm.recompile()
        eager = eager_gm(*args)
        if fused:
            assert torch.equal(eager, torch.ops.nb200.fold(args[0], 0, [0.0, 0.0, 1.0, 1.0, 1.0, 1.0], False, 1,
                                                           1024, 4))
            _check_against_oracle(name, args, eager, oracle_mod)
        ep.example_inputs = (tuple(args), {})  # the fixtures keep none; AOTInductor compiles from these
        pkg = A.compile_package(ep, str(tmp_path / f"{name}.pt2"))
        torch.save([t.cpu() for t in args], tmp_path / f"{name}.args.pt")
        jobs.append((name, pkg, eager))
    torch.cuda.synchronize()
    script = f"""
import sys, torch
import ctypes
ctypes.CDLL({os.path.join(ROOT, "neptune_opt_b200", "libneptune_b200_torch.so")!r}, mode=ctypes.RTLD_GLOBAL)
torch.ops.load_library({os.path.join(ROOT, "neptune_opt_b200", "libneptune_b200_torch.so")!r})
for name in {[j[0] for j in jobs]!r}:
    args = [t.cuda() for t in torch.load({str(tmp_path)!r} + "/" + name + ".args.pt")]
    runner = torch._inductor.aoti_load_package({str(tmp_path)!r} + "/" + name + ".pt2")
    out = runner(*args)
    out = list(out) if isinstance(out, (list, tuple)) else [out]
    torch.cuda.synchronize()
    torch.save([t.cpu() for t in out], {str(tmp_path)!r} + "/" + name + ".out.pt")
assert not any(m.startswith("neptune_opt_b200") for m in sys.modules)
assert not hasattr(torch.ops.neptune, "logsumexp_tiny0_b16384w0")
"""
    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    res = subprocess.run([sys.executable, "-c", script], cwd=str(tmp_path), env=env, capture_output=True, text=True,
                         timeout=900)
    assert res.returncode == 0, res.stderr[-3000:]
    for name, _pkg, eager in jobs:
        fresh = torch.load(tmp_path / f"{name}.out.pt")
        assert len(fresh) == 1, name
        assert torch.equal(fresh[0], eager.cpu()), f"{name}: the package differs from the eager rewrite"


def _reference_root():
    root = os.environ.get("NEPTUNE_REFERENCE") or os.path.join(ROOT, "baseline", "_ref")
    return root if os.path.isdir(os.path.join(root, "neptune_opt")) else None


def test_reference_apply_and_compile_best_drive_this_backend(tmp_path):
    root = _reference_root()
    if root is None:
        pytest.skip("the reference is not installed under baseline/_ref")
    code = f"""
import json, sys
sys.path[:0] = [{root!r}, {ROOT!r}, {GOLDEN!r}]
import torch, neptune_codegen, neptune_opt
from neptune_opt.ab import compile_best
import neptune_opt_b200 as NB
from neptune_opt_b200 import binding
import rewrite_models
binding.install(neptune_codegen)
# packages are compiled by the reference's own _package; give Inductor a host compiler that builds
# its OpenMP wrapper code (environment set-up, as for any AOTInductor user of this image)
import neptune_opt_b200.aot as A
torch._inductor.config.cpp.cxx = (None, A.host_compiler())
A.enable_c_shims()  # the packages call the nb200 ops through their C entry points
from neptune_opt_b200 import inductor_pass
inductor_pass.enable()  # 16-bit regions read their storage directly (widen/narrow casts folded in)
# bf16 outputs: the reference's explicit ULP slack (the ATen graph and the kernel round the same
# fp32 values; RMSNorm rounds twice)
ULPS = {{"rms_norm_bf16": 2, "logsumexp_split_bf16": 1}}
results = {{}}
for name, (cls, build, kwargs) in rewrite_models.CASES.items():
    args = build("cuda")
    ep = torch.export.export(cls(), args)
    slack = {{"max_ulps": ULPS[name]}} if name in ULPS else {{}}
    report = neptune_opt.apply(ep, verify_with=(cls(), args), **kwargs, **slack)
    targets = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    before = NB.launch_count()
    choice = compile_best(cls(), args, package_dir={str(tmp_path)!r} + "/" + name, verbose=False,
                          capabilities=kwargs.get("capabilities", ()), plans=(kwargs.get("plan", "serial"),),
                          reps=5, rounds=3, **slack)
    results[name] = {{"verified": bool(report.verified), "fusions": len(report.fusions),
                     "targets": targets, "fused_package": choice.fused_package,
                     "used_fusion": bool(choice.used_fusion), "reason": choice.reason,
                     "launches": NB.launch_count() - before, "speedup": choice.speedup}}
print(json.dumps(results))
"""
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=1800)
    assert res.returncode == 0, res.stderr[-3000:]
    results = json.loads(res.stdout.strip().splitlines()[-1])
    for name, r in results.items():
        assert r["verified"] and r["fusions"] == 1, (name, r)
        assert any(t.startswith("neptune.") for t in r["targets"]), (name, r)
        assert r["fused_package"], (name, r)  # compiled, loaded and matched the baseline's numbers
        assert r["launches"] > 0, (name, r)
        print(f"\n{name}: compile_best {r['reason']} (speedup {r['speedup']})")


def test_compile_best_keeps_the_fusion_at_the_benchmark_configurations(tmp_path):
    """The reference's compile_best (its export, apply, AOTInductor packaging, verification and
    A/B timing gate, neptune_opt/ab.py:270-530) on the benchmark configurations: logsumexp fp32
    [8192, 2048], RMSNorm bf16 [16384, 4096] and the split plan on bf16 [512, 262144]. The gate
    keeps a fused package only when it is faster than Inductor's own compilation of the
    unfused graph on that input."""
    root = _reference_root()
    if root is None:
        pytest.skip("the reference is not installed under baseline/_ref")
    code = f"""
import json, sys
sys.path[:0] = [{root!r}, {ROOT!r}, {GOLDEN!r}]
import torch, neptune_codegen
from neptune_opt.ab import compile_best
from neptune_opt_b200 import binding, inductor_pass
import neptune_opt_b200.aot as A
import rewrite_models as RM
binding.install(neptune_codegen)
torch._inductor.config.cpp.cxx = (None, A.host_compiler())
A.enable_c_shims()
inductor_pass.enable()
g = torch.Generator(device="cuda").manual_seed(7)
def lse():
    return (torch.randn(8192, 2048, device="cuda", generator=g) * 3.0,)
def rms():
    x = torch.randn(16384, 4096, device="cuda", generator=g).to(torch.bfloat16)
    return (x, (1 + 0.1 * torch.randn(4096, device="cuda", generator=g)).to(torch.bfloat16))
def split():
    return ((torch.randn(512, 262144, device="cuda", generator=g) * 3.0).to(torch.bfloat16),)
cases = {{
    "logsumexp_f32_8192x2048": (RM.LogsumexpRows, lse, {{}}, {{}}),
    "rms_norm_bf16_16384x4096": (RM.RmsNormGamma, rms, {{"capabilities": ("rms_norm",)}}, {{"max_ulps": 2}}),
    "logsumexp_split_bf16_512x262144": (RM.LogsumexpRows, split, {{"plan": "split"}}, {{"max_ulps": 1}}),
}}
out = {{}}
for name, (cls, build, kw, slack) in cases.items():
    choice = compile_best(cls(), build(), package_dir={str(tmp_path)!r} + "/" + name, verbose=False,
                          capabilities=kw.get("capabilities", ()), plans=(kw.get("plan", "serial"),), **slack)
    out[name] = {{"used_fusion": bool(choice.used_fusion), "speedup": choice.speedup, "reason": choice.reason}}
print(json.dumps(out))
"""
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=1800)
    assert res.returncode == 0, res.stderr[-3000:]
    results = json.loads(res.stdout.strip().splitlines()[-1])
    for name, r in results.items():
        print(f"\n{name}: speedup {r['speedup']:.2f} ({r['reason']})")
    for name, r in results.items():
        assert r["used_fusion"], (name, r)
