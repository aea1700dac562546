"""The reference's own front end rewriting graphs into this backend's ops, checked without a GPU.

tests/golden/rewrite_*.pt2 are ExportedPrograms that the reference's unchanged
`neptune_opt.apply` (neptune_opt/__init__.py:447-513) rewrote with this backend bound in
(`neptune_opt_b200.binding.install`), saved by tests/golden/make_rewrites.py. Here:
* each loads in a process without the reference, once the handles the rewrite used are registered,
  and holds the backend's per-key op where the reduction region was;
* AOTInductor's view of it -- the graph after decomposition -- holds only the C++-registered
  `nb200::*` ops, which a package calls by name without Python;
* where the reference is importable (its install under baseline/_ref, or NEPTUNE_REFERENCE), the
  fixtures are regenerated and must match: they are what the current reference produces.
"""
from __future__ import annotations

import json
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
ROOT = os.path.dirname(HERE)
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

with open(os.path.join(GOLDEN, "rewrites.json")) as _f:
    CASES = sorted(json.load(_f)["cases"])


def reference_root():
    for root in (os.environ.get("NEPTUNE_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if root and os.path.isdir(os.path.join(root, "neptune_opt")):
            return root
    return None


@pytest.mark.parametrize("name", CASES)
def test_rewritten_program_loads_and_holds_the_backend_op(name):
    from make_rewrites import load_case

    ep, case = load_case(name)
    targets = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert targets == case["targets"]
    ours = [t for t in targets if t.startswith("neptune.")]
    assert len(ours) == 1
    # the region's reduction ops are gone (the RMSNorm graph keeps the reference's unused stats
    # chain alive through its metadata assertions; nothing consumes it)
    if case["fusion"]["kind"] == "scalar":
        assert not any(t.startswith(("aten.exp", "aten.logsumexp", "aten.amax", "aten.sum", "aten.sqrt"))
                       for t in targets)


@pytest.mark.parametrize("name", CASES)
def test_decomposed_program_calls_only_cpp_registered_ops(name):
    from make_rewrites import load_case

    ep, _case = load_case(name)
    dec = ep.run_decompositions()
    targets = [str(n.target) for n in dec.graph.nodes if n.op == "call_function"]
    assert not any(t.startswith("neptune.") for t in targets), targets
    expected = {"logsumexp": "nb200.fold.default", "stable_l2": "nb200.fold.default",
                "rms_norm": "nb200.rms_norm.default", "segment_mean": "nb200.segment_pool.default"}
    assert expected[_case["fusion"]["skeleton"]] in targets


def test_fixtures_match_the_current_reference():
    root = reference_root()
    if root is None:
        pytest.skip("the reference is not installed here (baseline/_ref or NEPTUNE_REFERENCE)")
    import subprocess

    code = ("import json, sys; sys.path[:0] = [%r, %r, %r]\n"
            "import neptune_codegen, neptune_opt\n"
            "import make_rewrites as M, neptune_opt_b200 as NB\n"
            "from neptune_opt_b200 import binding\n"
            "from rewrite_models import CASES\n"
            "binding.install(neptune_codegen)\n"
            "out = {}\n"
            "for name in CASES:\n"
            "    ep, report, _ = M.rewrite_case(name, neptune_opt, [])\n"
            "    out[name] = [str(n.target) for n in ep.graph.nodes if n.op == 'call_function']\n"
            "print(json.dumps(out))\n") % (root, ROOT, GOLDEN)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    got = json.loads(res.stdout.strip().splitlines()[-1])
    with open(os.path.join(GOLDEN, "rewrites.json")) as f:
        want = {k: v["targets"] for k, v in json.load(f)["cases"].items()}
    assert got == want
