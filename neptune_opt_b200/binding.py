"""Bind this backend into an imported reference front end (the `neptune_codegen` package).

The reference's recogniser, rewrite transaction, `apply`, `preview` and `compile_best` reach the
backend only through names on the `neptune_codegen` package and two of its submodules:

* `neptune_recognize/rewrite.py:35`        `CG.autotune.best_config(...)`   (launch choice)
* `neptune_recognize/rewrite.py:171-175`   `neptune_codegen.template.validate_rms_inputs`,
                                           `neptune_codegen.torch_op.validate_segment_inputs`
* `neptune_recognize/rewrite.py:177`       `CG.state_op_handle(...)`
* `neptune_recognize/rewrite.py:182-185`   `CG.split_launch_shape(...)`, `CG.op_handle(...)`
* `neptune_opt/__init__.py:569`            `CG.op_handle(...)(x)`  (explicit op library)
* `neptune_codegen/__init__.py:72-77`      re-exports `run_rms_norm`, `run_segment_pool`,
                                           `as_state_op`, `split_launch_shape`, `MAX_SPLIT_PARTS`

`install(codegen)` points each of those names at this package, so the unchanged front end
registers and launches the sm_100a kernels instead of generating Triton. It is the programmatic
form of the one-module change a maintainer makes in the reference (`neptune_codegen/b200.py`
re-exporting these names); the recogniser's algebra (skeletons, certificates) stays the
reference's own. The returned callable restores the previous bindings.
"""
from __future__ import annotations

# (module attribute path relative to the neptune_codegen package, name in this package)
BINDINGS = (
    ("", "op_handle"), ("", "as_triton_op"), ("", "state_op_handle"), ("", "as_state_op"), ("", "run"),
    ("", "run_rms_norm"), ("", "run_segment_pool"), ("", "split_launch_shape"), ("", "MAX_SPLIT_PARTS"),
    ("", "autotune"), ("", "_TRITON_OPS"), ("", "triton_op_name"),
    ("template", "validate_rms_inputs"), ("template", "run"), ("template", "run_rms_norm"),
    ("template", "split_launch_shape"), ("template", "MAX_SPLIT_PARTS"),
    ("torch_op", "validate_segment_inputs"), ("torch_op", "op_handle"), ("torch_op", "as_triton_op"),
    ("torch_op", "state_op_handle"), ("torch_op", "as_state_op"), ("torch_op", "run_segment_pool"),
    ("torch_op", "_TRITON_OPS"), ("torch_op", "triton_op_name"),
)


def install(codegen):
    """Route the reference package `codegen` (an imported `neptune_codegen`) to this backend.

    Returns a function that undoes the routing."""
    import importlib

    import neptune_opt_b200 as NB

    saved = []
    for sub, name in BINDINGS:
        target = importlib.import_module(f"{codegen.__name__}.{sub}") if sub else codegen
        saved.append((target, name, getattr(target, name, None)))
        setattr(target, name, getattr(NB, name))

    def restore():
        for target, name, value in reversed(saved):
            setattr(target, name, value)

    return restore
