"""AOTInductor packaging of the region ops (torch.ops.nb200.*, registered from C++).

1. Each C++ op gives, bit for bit, the result of the Python layer's op over the same kernels.
2. A graph holding every region kind, exported and compiled by AOTInductor into a .pt2 package,
   reproduces the eager results bit for bit, and the package's calls launch this library's kernels.
3. A fresh process that loads only libneptune_b200_torch.so -- no neptune_opt_b200 Python code, no
   Python op registrations -- loads the package and gets the same results: the compiled regions
   need no Python op layer.
"""
from __future__ import annotations

import math
import os
import subprocess
import sys

import pytest

from conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCALE = 1.0 / math.sqrt(128)


def _inputs():
    import torch

    gen = torch.Generator().manual_seed(5)
    bf = torch.bfloat16
    x = (torch.randn(64, 2048, generator=gen) * 2).cuda()
    xb = torch.randn(32, 4096, generator=gen).to(bf).cuda()
    g = (1 + 0.1 * torch.randn(4096, generator=gen)).to(bf).cuda()
    wide = (torch.randn(8, 65536, generator=gen) * 3).to(bf).cuda()
    lengths = torch.poisson(torch.full((20,), 20.0), generator=gen).clamp(1, 200).long()
    data = torch.randn(int(lengths.sum()), 128, generator=gen).half().cuda()
    q, k, v = (torch.randn(1, 2, 300, 128, generator=gen).to(bf).cuda() for _ in range(3))
    return x, xb, g, wide, data, lengths.cuda(), q, k, v


def _regions_module():
    import torch

    import neptune_opt_b200.aot as A

    A.load()
    ops = torch.ops.nb200
    lse_p, l2_p = A.fold_params("logsumexp"), A.fold_params("stable_l2")

    class Regions(torch.nn.Module):
        def forward(self, x, xb, g, wide, data, lengths, q, k, v):
            a = ops.fold(x, 0, lse_p, False, 0, 0)
            b = ops.fold(x, 4, l2_p, True, 0, 0)
            y, l = ops.softmax(x, 0)
            n, nrm = ops.l2_normalize(xb)
            r = ops.rms_norm(xb, g, 1e-6)
            w = ops.fold(wide, 0, lse_p, False, 1, 16384)
            s = ops.segment_pool(data, lengths, False, 1, None, False)
            o, lse = ops.attention(q, k, v, True, SCALE)
            return a, b, y, l, n, nrm, r, w, s, o, lse

    return Regions()


def test_cpp_ops_match_the_python_layer_bitwise():
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200.aot as A

    x, xb, g, wide, data, lengths, q, k, v = _inputs()
    A.load()
    ops = torch.ops.nb200
    pairs = [
        (A.fold(x, "logsumexp"), NB.run("logsumexp", x)),
        (A.fold(x, "lse_scaled", {"T": 3.0}), NB.run("lse_scaled", x, T=3.0)),
        (A.fold(wide, "logsumexp", plan="split", block=16384), NB.run("logsumexp", wide, plan="split", block=16384)),
        (ops.softmax(x, 1)[0], NB.log_softmax(x)),
        (ops.l2_normalize(xb)[0], NB.l2_normalize(xb)),
        (ops.rms_norm(xb, g, 1e-6), NB.rms_norm(xb, g, 1e-6)),
        (ops.segment_pool(data, lengths, False, 1, None, False), NB.segment_mean(data, lengths)),
        (ops.attention(q, k, v, True, SCALE)[0], NB.attention(q, k, v, causal=True)),
    ]
    torch.cuda.synchronize()
    for i, (got, want) in enumerate(pairs):
        assert got.dtype == want.dtype and got.shape == want.shape, i
        assert torch.equal(got, want), f"pair {i} differs"
    assert ops.segment_status(torch.cuda.current_device(), True) == 0


def test_aoti_package_runs_the_regions(tmp_path):
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200.aot as A

    model = _regions_module()
    args = _inputs()
    eager = model(*args)
    ep = torch.export.export(model, args)
    # through the proxy executor's boxed calls, and (below) through the library's C shims
    boxed = torch._inductor.aoti_load_package(A.compile_package(ep, str(tmp_path / "boxed.pt2"), shims=False))
    for i, (a, b) in enumerate(zip(boxed(*args), eager)):
        assert torch.equal(a, b), f"output {i} of the boxed-call package differs from eager"
    pkg = A.compile_package(ep, str(tmp_path / "regions.pt2"))
    import zipfile

    wrapper = [n for n in zipfile.ZipFile(pkg).namelist() if n.endswith(".wrapper.cpp")]
    if wrapper:  # the package's generated code calls the C shims directly
        src = zipfile.ZipFile(pkg).read(wrapper[0]).decode()
        assert "aoti_torch_cuda_fold(" in src and "aoti_torch_cuda_attention(" in src
    runner = torch._inductor.aoti_load_package(pkg)
    before = NB.launch_count()
    got = runner(*args)
    torch.cuda.synchronize()
    assert NB.launch_count() > before, "the package did not launch this library's kernels"
    assert len(got) == len(eager)
    for i, (a, b) in enumerate(zip(got, eager)):
        assert torch.equal(a, b), f"output {i} of the package differs from eager"

    # a process with only the C++ registration: no neptune_opt_b200 import at all
    torch.save([t.cpu() for t in args], tmp_path / "args.pt")
    script = f"""
import torch
import ctypes
ctypes.CDLL({os.path.join(ROOT, "neptune_opt_b200", "libneptune_b200_torch.so")!r}, mode=ctypes.RTLD_GLOBAL)
torch.ops.load_library({os.path.join(ROOT, "neptune_opt_b200", "libneptune_b200_torch.so")!r})
args = [t.cuda() for t in torch.load({str(tmp_path / "args.pt")!r})]
runner = torch._inductor.aoti_load_package({str(pkg)!r})
out = runner(*args)
torch.cuda.synchronize()
assert not any(m.startswith("neptune_opt_b200") for m in __import__("sys").modules)
torch.save([t.cpu() for t in out], {str(tmp_path / "out.pt")!r})
"""
    env = {k: val for k, val in os.environ.items() if k != "PYTHONPATH"}
    res = subprocess.run([sys.executable, "-c", script], cwd=str(tmp_path), env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    fresh = torch.load(tmp_path / "out.pt")
    for i, (a, b) in enumerate(zip(fresh, eager)):
        assert torch.equal(a, b.cpu()), f"output {i} differs in the C++-only process"
