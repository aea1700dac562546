"""The C++-registered region ops (torch.ops.nb200.*) without a GPU: registration, schemas, shape
(Meta) kernels, and a torch.export trace of a graph holding every region kind -- the input an
AOTInductor package is compiled from."""
from __future__ import annotations

import pytest

SCHEMAS = {
    "fold": "nb200::fold(Tensor x, int skeleton, float[] params, bool keepdim, int plan, int block, "
            "int num_warps=0) -> Tensor",
    "softmax": "nb200::softmax(Tensor x, int mode) -> (Tensor, Tensor)",
    "l2_normalize": "nb200::l2_normalize(Tensor x) -> (Tensor, Tensor)",
    "rms_norm": "nb200::rms_norm(Tensor x, Tensor gamma, float eps) -> Tensor",
    "segment_pool": "nb200::segment_pool(Tensor data, Tensor segments, bool offsets, int reduce, float? initial, "
                    "bool unsafe) -> Tensor",
    "attention": "nb200::attention(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> (Tensor, Tensor)",
    "segment_status_word": "nb200::segment_status_word(int device) -> Tensor",
}


def _ops():
    import torch

    import neptune_opt_b200.aot as A

    A.load()
    return torch.ops.nb200


def test_cpp_ops_register_with_their_schemas():
    ops = _ops()
    for name, schema in SCHEMAS.items():
        assert str(getattr(ops, name).default._schema) == schema


def test_meta_kernels_compute_shapes_only():
    import torch

    import neptune_opt_b200.aot as A

    ops = _ops()
    meta = lambda *s, dt=torch.float32: torch.empty(*s, dtype=dt, device="meta")  # noqa: E731
    x = meta(4, 5, 300)
    assert A.fold(x, "logsumexp").shape == (4, 5)
    assert A.fold(x, "stable_l2", keepdim=True).shape == (4, 5, 1)
    y, lse = ops.softmax(x, 1)
    assert y.shape == x.shape and lse.shape == (4, 5)
    assert ops.rms_norm(meta(7, 64, dt=torch.bfloat16), meta(64, dt=torch.bfloat16), 1e-6).shape == (7, 64)
    assert ops.segment_pool(meta(100, 3, 8), meta(11, dt=torch.int64), True, 0, None, False).shape == (10, 3, 8)
    assert ops.segment_pool(meta(100, 8), meta(11, dt=torch.int64), False, 1, 0.5, False).shape == (11, 8)
    o, l = ops.attention(*(meta(2, 3, 300, 128, dt=torch.bfloat16) for _ in range(3)), True, 0.1)
    assert o.shape == (2, 3, 300, 128) and l.shape == (2, 3, 300) and l.dtype == torch.float32


def test_fold_params_follow_the_skeleton_defaults_and_domains():
    import neptune_opt_b200.aot as A

    assert A.fold_params("lse_scaled") == [0.0, 0.0, 2.0, 1.0, 1.0, 1.0]  # reference default T = 2
    assert A.fold_params("softcap_lse", {"beta": 0.3})[3] == 0.3
    with pytest.raises(NotImplementedError):
        A.fold_params("lse_scaled", {"T": -1.0})


def test_export_traces_every_region_kind():
    import torch

    import neptune_opt_b200.aot as A

    ops = _ops()

    class Regions(torch.nn.Module):
        def forward(self, x, xb, g, data, lengths, q, k, v):
            a = ops.fold(x, 0, A.fold_params("logsumexp"), False, 0, 0)
            y, l = ops.softmax(x, 0)
            n, nrm = ops.l2_normalize(x)
            r = ops.rms_norm(xb, g, 1e-6)
            s = ops.segment_pool(data, lengths, False, 1, None, False)
            o, lse = ops.attention(q, k, v, True, 0.08838834764831845)
            w = ops.fold(xb, 0, A.fold_params("logsumexp"), False, 1, 1024)
            return a, y, l, n, nrm, r, s, o, lse, w

    bf = torch.bfloat16
    args = (torch.randn(8, 300), torch.randn(8, 4096).to(bf), torch.ones(4096).to(bf), torch.randn(50, 16).half(),
            torch.full((5,), 10, dtype=torch.int64), *(torch.randn(1, 2, 256, 128).to(bf) for _ in range(3)))
    ep = torch.export.export(Regions(), args)
    targets = [str(n.target) for n in ep.graph.nodes if n.op == "call_function" and "nb200" in str(n.target)]
    assert targets == ["nb200.fold.default", "nb200.softmax.default", "nb200.l2_normalize.default",
                       "nb200.rms_norm.default", "nb200.segment_pool.default", "nb200.attention.default",
                       "nb200.fold.default"]


def test_cpp_ops_have_no_cpu_fallback():
    import torch

    ops = _ops()
    with pytest.raises((NotImplementedError, RuntimeError)):
        ops.fold(torch.randn(4, 8), 0, [0.0, 0.0, 1.0, 1.0, 1.0, 1.0], False, 0, 0)


def test_host_compiler_for_packages_builds_openmp_code():
    import neptune_opt_b200.aot as A

    assert A._cxx_builds_openmp(A.host_compiler())
