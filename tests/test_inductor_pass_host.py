"""The cast-fusion pass on graphs traced with fake tensors (no GPU): which region graphs it rewrites
and which it must leave alone. The numerics of the rewritten graphs run in
tests/test_reference_rewrites_gpu.py."""
from __future__ import annotations

import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def ops():
    import torch

    import neptune_opt_b200.aot as A

    try:
        A.load()
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"the C++ op library is not built: {e}")
    return torch.ops.nb200, A.fold_params("logsumexp")


def _trace(fn, *shapes_dtypes):
    import torch
    from torch.fx.experimental.proxy_tensor import make_fx

    args = [torch.empty(s, dtype=d, device="meta") for s, d in shapes_dtypes]
    return make_fx(fn, tracing_mode="fake")(*args)


def _targets(gm):
    return [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("plan,block", [(0, 0), (1, 1024)])
def test_widen_fold_narrow_becomes_one_fold_of_the_storage(ops, dtype, plan, block):
    import torch

    from neptune_opt_b200.inductor_pass import fuse_casts

    nb, p = ops
    dt = getattr(torch, dtype)

    def f(x):
        return nb.fold(x.float(), 0, p, False, plan, block, 0).to(dt)

    gm = _trace(f, ((8, 4096), dt))
    assert _targets(gm).count("aten._to_copy.default") == 2
    assert fuse_casts(gm.graph) == 1
    gm.graph.lint()
    gm.recompile()
    assert _targets(gm) == ["nb200.fold.default"]
    (fold,) = [n for n in gm.graph.nodes if n.op == "call_function"]
    assert fold.args[0].op == "placeholder" and fold.args[1:6] == (0, p, False, plan, block)
    assert fold.meta["val"].dtype == dt and tuple(fold.meta["val"].shape) == (8,)


def test_prims_convert_element_type_form_is_matched(ops):
    import torch

    from neptune_opt_b200.inductor_pass import fuse_casts

    nb, p = ops
    cvt = torch.ops.prims.convert_element_type.default

    def f(x):
        return cvt(nb.fold(cvt(x, torch.float32), 0, p, True, 0, 0, 0), torch.bfloat16)

    gm = _trace(f, ((4, 512), torch.bfloat16))
    assert fuse_casts(gm.graph) == 1
    assert _targets(gm) == ["nb200.fold.default"]


def test_graphs_whose_result_differs_are_left_alone(ops):
    import torch

    from neptune_opt_b200.inductor_pass import fuse_casts

    nb, p = ops
    bf = torch.bfloat16

    def fp32_result_used(x):  # the float32 result feeds other arithmetic
        y = nb.fold(x.float(), 0, p, False, 0, 0, 0)
        return y.to(bf), y * 2

    def other_dtype_out(x):  # narrowed to a dtype other than the storage's: two roundings differ
        return nb.fold(x.float(), 0, p, False, 0, 0, 0).to(torch.float16)

    def fp32_input(x):  # nothing to fold away
        return nb.fold(x, 0, p, False, 0, 0, 0).to(bf)

    def not_narrowed(x):  # a float32 output is the user's
        return nb.fold(x.float(), 0, p, False, 0, 0, 0)

    def widened_to_f64(x):
        return nb.fold(x.double().float(), 0, p, False, 0, 0, 0).to(bf)

    cases = [(fp32_result_used, bf), (other_dtype_out, bf), (fp32_input, torch.float32),
             (not_narrowed, bf), (widened_to_f64, bf)]
    for fn, dt in cases:
        gm = _trace(fn, ((8, 256), dt))
        before = _targets(gm)
        assert fuse_casts(gm.graph) == 0, fn.__name__
        assert _targets(gm) == before, fn.__name__


def test_the_widened_input_stays_when_another_node_reads_it(ops):
    import torch

    from neptune_opt_b200.inductor_pass import fuse_casts

    nb, p = ops

    def f(x):
        w = x.float()
        return nb.fold(w, 0, p, False, 0, 0, 0).to(torch.bfloat16), w.sum()

    gm = _trace(f, ((8, 256), torch.bfloat16))
    assert fuse_casts(gm.graph) == 1
    gm.graph.lint()
    targets = _targets(gm)
    assert targets.count("aten._to_copy.default") == 1 and "nb200.fold.default" in targets


def test_reference_rewrite_of_a_bf16_split_fold_is_fused(ops):
    """The reference front end's own rewrite (a fixture): widen, per-key split op, narrow. Exported
    for packaging it decomposes to nb200.fold between the casts, which the pass folds."""
    if GOLDEN not in sys.path:
        sys.path.insert(0, GOLDEN)
    from make_rewrites import load_case

    from neptune_opt_b200.inductor_pass import fuse_casts

    ep, _case = load_case("logsumexp_split_bf16")
    gm = ep.run_decompositions().module()
    assert _targets(gm) == ["aten._to_copy.default", "nb200.fold.default", "aten._to_copy.default"]
    assert fuse_casts(gm.graph) == 1
    assert _targets(gm) == ["nb200.fold.default"]
    ep32, _ = load_case("logsumexp_f32")
    gm32 = ep32.run_decompositions().module()
    assert fuse_casts(gm32.graph) == 0


def test_enable_installs_the_pass_once_after_an_existing_one(ops):
    import torch._inductor.config as cfg

    from neptune_opt_b200 import inductor_pass

    calls = []

    class Earlier:
        def __call__(self, graph):
            calls.append(graph)

        def uuid(self):
            return "earlier"

    with cfg.patch({"post_grad_custom_post_pass": Earlier()}):
        installed = inductor_pass.enable()
        assert inductor_pass.enable() is installed
        assert "earlier" in installed.uuid() and inductor_pass.VERSION in installed.uuid()
        import torch.fx

        installed(torch.fx.Graph())
        assert len(calls) == 1
