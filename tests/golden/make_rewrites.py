"""Generate the rewritten-program fixtures: the reference's own front end driving this backend.

    python tests/golden/make_rewrites.py [REFERENCE_ROOT]     (default: $NEPTUNE_REFERENCE)

Needs the reference (Defyli/neptune-opt, pure Python) importable from REFERENCE_ROOT; needs no GPU.
For every case of rewrite_models.CASES it
  1. exports the module with torch.export on fake CUDA tensors of the case's shapes/dtypes;
  2. binds this backend into the reference (`neptune_opt_b200.binding.install(neptune_codegen)`)
     and runs the reference's unchanged `neptune_opt.apply(ep, **kwargs)`
     (neptune_opt/__init__.py:447-513 -> neptune_recognize/rewrite.py:159-217 -> our op_handle /
     state_op_handle), which rewrites the graph in place;
  3. saves the rewritten ExportedProgram as rewrite_<case>.pt2 and records in rewrites.json the
     handle calls the rewrite made (so a loader can register the same ops before loading), the
     reference's fusion report and the op targets of the rewritten graph.
The tests load these programs without the reference and run them on the GPU, eagerly and as
AOTInductor packages.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
MANIFEST = os.path.join(HERE, "rewrites.json")


def rewrite_case(name, neptune_opt, record):
    """Export + the reference's apply for one case; returns (ep, report, handle calls)."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    from rewrite_models import CASES

    cls, build, kwargs = CASES[name]
    real = build("cpu")
    with FakeTensorMode(allow_non_fake_inputs=True):
        fake = tuple(torch.empty(t.shape, dtype=t.dtype, device="cuda") for t in real)
    ep = torch.export.export(cls(), fake)
    record.clear()
    report = neptune_opt.apply(ep, **kwargs)
    return ep, report, list(record)


def main(reference_root: str) -> None:
    import torch

    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    sys.path.insert(0, reference_root)
    import neptune_codegen
    import neptune_opt

    import neptune_opt_b200 as NB
    from neptune_opt_b200 import binding
    from rewrite_models import CASES

    binding.install(neptune_codegen)
    record = []

    def recorded(kind, fn):
        def wrapper(*args, **kwargs):
            record.append({"kind": kind, "args": list(args), "kwargs": kwargs})
            return fn(*args, **kwargs)
        return wrapper

    neptune_codegen.op_handle = recorded("op_handle", NB.op_handle)
    neptune_codegen.state_op_handle = recorded("state_op_handle", NB.state_op_handle)

    manifest = {"torch": torch.__version__, "cases": {}}
    for name in CASES:
        ep, report, calls = rewrite_case(name, neptune_opt, record)
        if len(report.fusions) != 1 or not report.graph_changed:
            raise RuntimeError(f"{name}: the reference did not rewrite exactly one region: {report}")
        path = os.path.join(HERE, f"rewrite_{name}.pt2")
        ep._example_inputs = None  # fake CUDA tensors of the export: nothing worth keeping
        torch.export.save(ep, path)
        targets = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
        fusion = report.fusions[0]
        manifest["cases"][name] = {
            "file": os.path.basename(path), "handles": calls, "targets": targets,
            "fusion": {"skeleton": fusion.skeleton, "params": fusion.params, "plan": fusion.plan,
                       "kind": fusion.kind, "operation": fusion.operation},
        }
        print(f"{name}: {fusion.skeleton} ({fusion.plan}) -> {[t for t in targets if 'neptune' in t]}")
    with open(MANIFEST, "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
        f.write("\n")


def register_handles(case: dict) -> None:
    """Register, in this process, the ops a fixture's rewrite created (before torch.export.load)."""
    import neptune_opt_b200 as NB

    for call in case["handles"]:
        fn = {"op_handle": NB.op_handle, "state_op_handle": NB.state_op_handle}[call["kind"]]
        kwargs = dict(call["kwargs"])
        if "params" in kwargs and isinstance(kwargs["params"], dict):
            kwargs["params"] = dict(kwargs["params"])
        fn(*call["args"], **kwargs)


def load_case(name: str):
    """(rewritten ExportedProgram, manifest entry) of fixture `name`."""
    import torch

    with open(MANIFEST) as f:
        case = json.load(f)["cases"][name]
    register_handles(case)
    return torch.export.load(os.path.join(HERE, case["file"])), case


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["NEPTUNE_REFERENCE"])
