"""Host-side contracts of the backend, mirroring the reference's CPU tests of the same API:
metadata (meta/Fake) shapes without launches, the runtime input contract and its exception types,
split capacity, op identity/registration with Fake kernels, export with dynamic batch, and the
launch policy. None of these launch a kernel."""
from __future__ import annotations

import pytest
import torch

import neptune_opt_b200 as NB
from neptune_opt_b200 import autotune, template, torch_op


def test_supported_set_and_defaults_mirror_the_reference():
    assert NB.supported() == sorted(["decay_renorm", "linear_attn", "logsumexp", "lse_biased", "lse_scaled",
                                     "rmsnorm_max", "softcap_lse", "stable_l2", "std", "sumsq_div", "variance"])
    assert NB.param_defaults("lse_scaled") == {"T": 2.0, "tiny": 0.0}
    assert NB.param_defaults("lse_biased") == {"alpha": 1.0, "tiny": 0.0}
    assert NB.param_defaults("rmsnorm_max") == {"eps": 1.0}
    assert NB.op_parameters("lse_biased") == ("alpha",)
    with pytest.raises(TypeError, match="alpha"):
        NB.lse_biased(torch.empty(2, 8, device="meta"))


def test_runtime_rejects_unsupported_inputs_but_meta_infers_shapes():
    cases = [(torch.empty(2, 8), ValueError, "device"),
             (torch.empty((), device="meta"), ValueError, "rank"),
             (torch.empty(2, 0, device="meta"), RuntimeError, "width"),
             (torch.empty(2, 8, device="meta", dtype=torch.float64), TypeError, "dtype"),
             (torch.empty(2, 8, device="meta", dtype=torch.int32), TypeError, "dtype")]
    for x, error, message in cases:
        with pytest.raises(error, match=message):
            NB.run("logsumexp", x)
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        for shape in ((8,), (2, 3, 8), (2, 0, 8)):
            for keep in (False, True):
                out = NB.run("logsumexp", torch.empty(shape, device="meta", dtype=dtype), keepdim=keep)
                assert out.shape == shape[:-1] + ((1,) if keep else ())
                assert out.dtype == dtype


def test_split_capacity_power_of_two_and_concrete_width():
    assert NB.split_launch_shape(1025, 1024) == (2, 2)
    assert NB.split_launch_shape(4096, 1) == (4096, 4096)
    with pytest.raises(NotImplementedError, match="capacity"):
        NB.split_launch_shape(4097, 1)
    with pytest.raises(ValueError, match="power of two"):
        NB.split_launch_shape(32, 3)

    class SymbolicWidth:
        def __int__(self):
            raise AssertionError("must not concretise symbolic width")

    with pytest.raises(NotImplementedError, match="concrete width"):
        NB.split_launch_shape(SymbolicWidth(), 1024)
    with pytest.raises(NotImplementedError, match="two_pass"):
        NB.run("variance", torch.empty(2, 8, device="meta"), plan="split")
    for shape in ((17,), (3, 17), (2, 3, 17)):
        x = torch.empty(shape, device="meta", dtype=torch.bfloat16)
        for plan in ("serial", "split"):
            for keep in (False, True):
                out = NB.run("stable_l2", x, block=8, keepdim=keep, plan=plan)
                assert out.shape == shape[:-1] + ((1,) if keep else ())


def test_parameter_domains_follow_the_certificate():
    with pytest.raises(NotImplementedError, match="positive"):
        NB.run("lse_scaled", torch.empty(2, 8, device="meta"), T=-1.0)
    with pytest.raises(NotImplementedError, match="finite"):
        NB.run("lse_biased", torch.empty(2, 8, device="meta"), alpha=float("inf"))
    with pytest.raises(NotImplementedError, match="nonnegative"):
        NB.run("logsumexp", torch.empty(2, 8, device="meta"), tiny=-1.0)


def test_rms_contract_validation_and_capacity():
    def meta(shape, dtype=torch.float32):
        return torch.empty(shape, device="meta", dtype=dtype)

    cases = [
        (meta(()), meta((1,)), ValueError, "rank"),
        (meta((2, 0)), meta((0,)), RuntimeError, "width"),
        (meta((2, 8), torch.uint8), meta((8,), torch.uint8), TypeError, "dtype"),
        (meta((2, 8), torch.float16), meta((8,)), ValueError, "dtype/device"),
        (meta((2, 8)), meta((1, 8)), ValueError, "1D"),
        (meta((2, 8)), meta((7,)), RuntimeError, "width"),
    ]
    for x, gamma, error, message in cases:
        with pytest.raises(error, match=message):
            NB.run_rms_norm(x, gamma)
    with pytest.raises(ValueError, match="CUDA"):
        NB.run_rms_norm(torch.empty(2, 8), torch.empty(8))
    for width, plan in ((32768, "serial"), (32769, "split"), (4194304, "split")):
        assert NB.validate_rms_inputs(meta((0, width)), meta((width,)), {"eps": 1e-6}, plan=plan,
                                      metadata=True) == (0, width)
    for width, plan, message in ((32769, "serial", "32768"), (4194305, "split", "capacity")):
        with pytest.raises(NotImplementedError, match=message):
            NB.validate_rms_inputs(meta((0, width)), meta((width,)), {"eps": 1e-6}, plan=plan, metadata=True)
    for eps in (True, "1e-6", None, 0, -1, float("inf"), float("nan")):
        with pytest.raises(ValueError, match="eps"):
            NB.run_rms_norm(meta((2, 8)), meta((8,)), eps=eps)
    x = torch.empty(512, 2, device="meta").t()
    out = NB.run_rms_norm(x, torch.empty(512, device="meta"))
    assert out.stride() == (512, 1)


def test_op_handles_are_overloads_with_fake_kernels_and_export():
    from torch._subclasses.fake_tensor import FakeTensorMode

    op = NB.as_cuda_op("logsumexp", lib="nb200_cpu_metadata", keepdim=True)
    handle = NB.op_handle("logsumexp", lib="nb200_cpu_metadata", keepdim=True)
    assert isinstance(handle, torch._ops.OpOverload)
    assert NB.as_triton_op is NB.as_cuda_op
    with FakeTensorMode():
        for shape in ((8,), (2, 3, 8), (0, 3, 8)):
            out = op(torch.empty(shape, dtype=torch.bfloat16))
            assert out.shape == shape[:-1] + (1,)
            assert out.dtype == torch.bfloat16

    class Model(torch.nn.Module):
        def forward(self, x):
            return op(x)

    exported = torch.export.export(Model(), (torch.empty(2, 3, 8),),
                                   dynamic_shapes={"x": {0: torch.export.Dim("batch", min=1, max=16)}})
    node = next(n for n in exported.graph.nodes if n.op == "call_function")
    assert isinstance(node.meta["val"].shape[0], torch.SymInt)


def test_op_identity_carries_parameters_rank_config_and_plan():
    a = NB.as_cuda_op("lse_scaled", lib="nb200_ident", params={"T": 2.0})
    b = NB.as_cuda_op("lse_scaled", lib="nb200_ident", params={"T": 3.0})
    c = NB.as_cuda_op("lse_scaled", lib="nb200_ident", params={"T": 2.0}, keepdim=True)
    d = NB.as_cuda_op("lse_scaled", lib="nb200_ident", params={"T": 2.0}, plan="split")
    assert len({a.__name__, b.__name__, c.__name__, d.__name__}) == 4
    assert NB.as_cuda_op("lse_scaled", lib="nb200_ident", params={"T": 2.0}) is a
    assert autotune.op_key("neptune", "logsumexp", {"tiny": 0.0}, False, 1024, 4) == "neptune::logsumexp_tiny0_b1024w4"


def test_state_and_segment_ops_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    rms = NB.state_op_handle("rms_norm", {"eps": 1e-6}, lib="nb200_state_meta")
    assert isinstance(rms, torch._ops.OpOverload)
    seg = NB.as_segment_op("segment_mean", {"initial": -2.0}, lib="nb200_seg_meta")
    assert isinstance(NB.segment_op_handle("segment_mean", {"initial": -2.0}, lib="nb200_seg_meta"),
                      torch._ops.OpOverload)
    with FakeTensorMode():
        assert rms(torch.empty(3, 8), torch.empty(8)).shape == (3, 8)
        assert seg(torch.empty(3, 0), torch.empty(2, dtype=torch.int64)).shape == (2, 0)
        assert seg(torch.empty(0, 3), torch.empty(0, dtype=torch.int64)).shape == (0, 3)
    with pytest.raises(ValueError, match="unknown segment parameters"):
        NB.as_segment_op("segment_sum", {"bogus": 1})
    with pytest.raises(NotImplementedError, match="ordered"):
        NB.as_segment_op("segment_sum", {}, plan="split")
    with pytest.raises(TypeError, match="index dtype"):
        NB.validate_segment_inputs(torch.empty(3, 2, device="meta"), torch.empty(2, device="meta"), metadata=True)
    with pytest.raises(RuntimeError, match="overflow"):
        NB.validate_segment_inputs(torch.empty(3, 2, device="meta", dtype=torch.float16),
                                   torch.empty(2, device="meta", dtype=torch.int64), initial=1e6, metadata=True)
    out = NB.run_segment_pool(torch.empty(7, 4, device="meta"), torch.empty(3, dtype=torch.int64, device="meta"))
    assert out.shape == (3, 4)


def test_segment_status_messages_follow_reference_order():
    with pytest.raises(RuntimeError, match="nonnegative and within data bounds"):
        torch_op.check_segment_status(1 | 4)
    with pytest.raises(RuntimeError, match="sum to data axis0"):
        torch_op.check_segment_status(2)
    with pytest.raises(RuntimeError, match="monotonic"):
        torch_op.check_segment_status(8)
    torch_op.check_segment_status(0)
    assert torch_op._initial_bits(-0.0) == 0x80000000
    assert torch_op._initial_bits(None) == 0


def test_launch_policy_defaults_and_table():
    assert autotune.best_config(8192, 2048, torch.float32) == (16384, 0)
    assert autotune.best_config(16384, 4096, torch.bfloat16) == (16384, 0)
    assert autotune.best_config(4, 100, torch.float32, device="cpu") == (16384, 0)
    assert autotune.launch_for((16384, 0)) is None
    assert autotune.machine_key("NVIDIA B200") == "b200"
    assert autotune.shape_key(1, 262144) == ("single", 262144)
    assert autotune.launch_for((16384, 1)).variant == 1
    assert autotune.launch_for((16384, 8)).threads == 256
    for entry in autotune.tables().values():
        for cfg in entry["table"].values():
            assert cfg in autotune.CANDIDATES
    res = [autotune.Result(16384, 0, 1.0), autotune.Result(16384, 8, 0.97)]
    assert autotune.choose(res, (16384, 0))[0] == (16384, 0)
    res = [autotune.Result(16384, 0, 1.0), autotune.Result(16384, 8, 0.5)]
    assert autotune.choose(res, (16384, 0))[0] == (16384, 8)


def test_launch_policy_bucket_choice_and_table_writer(tmp_path):
    R = autotune.Result
    # a bucket's choice is the best WORST-CASE gain over its shapes, and must clear the noise bar
    runs = [[R(16384, 0, 1.0), R(16384, 8, 0.5), R(4096, 1, 0.9)],
            [R(16384, 0, 1.0), R(16384, 8, 0.93), R(4096, 1, 0.8)]]
    cfg, worst, why = autotune.choose_many(runs)
    assert cfg == (4096, 1) and abs(worst - 1.0 / 0.9) < 1e-9 and "worst case" in why
    flat = [[R(16384, 0, 1.0), R(16384, 8, 0.97)], [R(16384, 0, 1.0), R(16384, 8, 0.5)]]
    assert autotune.choose_many(flat)[0] == autotune.DEFAULT
    assert autotune.choose_many([[R(16384, 8, 1.0)]])[0] == autotune.DEFAULT  # default unmeasured
    # a written table round-trips through the module loader and only keeps known candidates
    merged = autotune.merge_table(autotune.tables(), "test-gpu", "a test",
                                  {("few", 4096): (16384, 8), ("many", 256): (3, 3)})
    path = tmp_path / "launch_table.py"
    autotune.write_tables(str(path), merged)
    ns = {}
    exec(path.read_text(), ns)
    assert ns["TABLES"]["test-gpu"]["table"] == {("few", 4096): (16384, 8)}
    assert ns["TABLES"]["test-gpu"]["measured_on"] == "a test"
    assert set(ns["TABLES"]) == set(autotune.tables()) | {"test-gpu"}
    # the campaign covers every rows class at every width bucket it names, within its size cap
    shapes = autotune.campaign_shapes()
    assert {autotune.rows_class(r) for r, _ in shapes} == {"single", "few", "many"}
    assert all(r * c <= max(autotune.CAMPAIGN_MAX_ELEMS, c * autotune.THIN_ROWS) for r, c in shapes)
    assert {c for _, c in shapes} == set(autotune.CAMPAIGN_WIDTHS)


def test_template_helpers():
    assert template.dtype_code(torch.bfloat16) == 1
    x = torch.randn(2, 3, 8)
    flat, rows, ncols = template._row_last_layout(x)
    assert (rows, ncols) == (6, 8) and flat.data_ptr() == x.data_ptr()
