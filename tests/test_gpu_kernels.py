"""GPU parity of the sm_100a kernels against the CPU oracle and the reference's golden vectors.

Tolerances: fp32 results within rtol 1e-5 (plus a cancellation floor of 1e-6 x
the batch's largest magnitude for the sum-of-ratios skeletons); bf16/fp16 results within 1 ulp of
the oracle's fp32 value; nonfinite values identical; RMSNorm as `assert_rms_close`; segment
pooling and span construction bit-exact.
"""
from __future__ import annotations

import ast
import ctypes

import numpy as np
import pytest

from conftest import (assert_close_dtype, assert_nonfinite_equal, assert_rms_close, cuda_available, golden,
                      round_to)

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

DTYPES = ("float32", "bfloat16", "float16")
TEST_PARAMS = {"lse_biased": {"alpha": -0.75}, "lse_scaled": {"T": 3.0}, "softcap_lse": {"beta": 0.3},
               "decay_renorm": {"N": 2.5}, "rmsnorm_max": {"eps": 1e-6}, "logsumexp": {"tiny": 0.0}}


def _t(dtype):
    import torch

    return getattr(torch, dtype)


def _inputs(dtype, gen):
    """(label, tensor) cases: contiguous narrow/wide rows, ragged widths, strided/transposed/expanded
    views and rank 3, covering the warp-per-row, CTA-per-row, vector and scalar-load paths."""
    import torch

    dt = _t(dtype)
    cases = []
    for shape in ((37, 1000), (64, 2048), (5, 3000), (9, 17), (3, 70000), (1, 262144), (200, 96)):
        cases.append((f"contig{shape}", (torch.randn(*shape, generator=gen) * 2.0).to(dt).cuda()))
    base = (torch.randn(12, 2050, generator=gen) * 2.0).to(dt).cuda()
    cases.append(("col_stride2", base[:, ::2]))
    cases.append(("transposed", (torch.randn(300, 40, generator=gen) * 2).to(dt).cuda().t()))
    cases.append(("expanded", (torch.randn(6, 1, generator=gen)).to(dt).cuda().expand(6, 500)))
    cases.append(("rank3", (torch.randn(4, 5, 777, generator=gen) * 2).to(dt).cuda()))
    cases.append(("offset_unaligned", (torch.randn(8 * 1001 + 1, generator=gen)).to(dt).cuda()[1:].view(8, 1001)))
    return cases


def _oracle_rows(x):
    return x.float().reshape(-1, x.shape[-1]).cpu().numpy()


def _sum_floor(name, rows, params):
    """Cancellation floor of the signed-sum skeletons (linear_attn: terms x / max|x|; decay_renorm:
    x / (N + max|x|)): 2^-19 sqrt(sum t^2) per row. The rounding errors of an fp32 sum of N such
    terms form a random walk of about 2^-24 sqrt(log2 N) sqrt(sum t^2) in any summation order, so a
    result that cancels to near zero is compared at that scale (the floor is ~8 times it), not
    relative to itself. Other skeletons sum terms of one sign: no floor."""
    if name not in ("linear_attn", "decay_renorm"):
        return 0.0
    a = np.asarray(rows, np.float64)
    den = np.abs(a).max(axis=1) + (params.get("N", 0.0) if name == "decay_renorm" else 0.0)
    t = a / np.maximum(den, 1e-30)[:, None]
    return float(np.max(np.sqrt((t * t).sum(axis=1)))) * 2.0 ** -19


def _scale(ref):
    fin = np.isfinite(ref)
    return float(np.max(np.abs(ref[fin]))) if fin.any() else 0.0


@pytest.mark.parametrize("name", ["logsumexp", "lse_biased", "lse_scaled", "softcap_lse", "stable_l2",
                                  "linear_attn", "decay_renorm", "sumsq_div", "rmsnorm_max", "variance", "std"])
def test_serial_fold_matches_oracle_all_layouts_and_dtypes(name, oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(7)
    params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
    for dtype in DTYPES:
        for label, x in _inputs(dtype, gen):
            for keep in (False, True):
                out = NB.run(name, x, keepdim=keep, **params)
                assert out.dtype == x.dtype and out.shape == x.shape[:-1] + ((1,) if keep else ())
            ref = oracle_mod.fold(name, _oracle_rows(x), params)
            got = out.float().reshape(-1).cpu().numpy()
            assert_close_dtype(got, ref, dtype, atol32=1e-6 * (1 + _scale(ref)))


@pytest.mark.parametrize("cfg", [(16384, 0), (16384, 1), (16384, 4), (16384, 8), (4096, 16)])
def test_every_launch_variant_agrees(cfg, oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(3)
    for name in ("logsumexp", "stable_l2", "rmsnorm_max", "std"):
        params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
        for shape in ((33, 777), (7, 20000)):
            for dtype in ("float32", "bfloat16"):
                x = (torch.randn(*shape, generator=gen) * 2).to(_t(dtype)).cuda()
                out = NB.run(name, x, block=cfg[0], num_warps=cfg[1], **params)
                ref = oracle_mod.fold(name, _oracle_rows(x), params)
                assert_close_dtype(out.float().cpu().numpy(), ref, dtype, atol32=1e-6 * (1 + _scale(ref)))


def test_log_family_nonfinite_rows_exact(oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    rows = golden("fold.npz")["logsumexp|0|special|float32|x"]
    wide = np.full((rows.shape[0], 3000), -np.inf, np.float32)
    wide[:, :7] = rows
    wide[[3, 5, 7], 7:] = 0.25
    for name in ("logsumexp", "lse_biased", "lse_scaled", "softcap_lse"):
        params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
        for data in (rows, wide):
            for dtype in DTYPES:
                x = torch.from_numpy(data).to(_t(dtype)).cuda()
                for plan, block in (("serial", None), ("split", 1024)):
                    out = NB.run(name, x, plan=plan, block=block, **params).float().cpu().numpy()
                    ref = oracle_mod.fold(name, x.float().cpu().numpy(), params)
                    assert_nonfinite_equal(out, ref)
                    assert_close_dtype(out, ref, dtype)


def test_fold_matches_reference_golden_vectors():
    import torch

    import neptune_opt_b200 as NB

    data = golden("fold.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in data.files})
    for key in keys:
        name, _pi, _label, dtype = key.split("|")
        params = dict(ast.literal_eval(str(data[key + "|params"])))
        x = torch.from_numpy(data[key + "|x"]).to(_t(dtype)).cuda()
        ref = data[key + "|serial"]
        scale = _scale(ref)
        got = NB.run(name, x, **params).float().cpu().numpy()
        assert_close_dtype(got, ref, dtype, atol32=1e-6 * (1 + scale))
        if key + "|split" in data.files:
            block = int(data[key + "|split_block"])
            got2 = NB.run(name, x, plan="split", block=block, **params).float().cpu().numpy()
            assert_close_dtype(got2, data[key + "|split"], dtype, atol32=1e-6 * (1 + scale))


@pytest.mark.parametrize("block", [128, 1024, 16384])
def test_split_plan_matches_oracle(block, oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(11)
    for name in ("logsumexp", "lse_scaled", "stable_l2", "linear_attn", "decay_renorm", "sumsq_div",
                 "rmsnorm_max", "softcap_lse", "lse_biased"):
        params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
        for shape in ((16, 70000), (3, 262144), (40, 5000)):
            if -(-shape[1] // block) > NB.MAX_SPLIT_PARTS:
                continue
            for dtype in DTYPES:
                x = (torch.randn(*shape, generator=gen) * 3).to(_t(dtype)).cuda()
                out = NB.run(name, x, plan="split", block=block, **params)
                ref = oracle_mod.fold(name, _oracle_rows(x), params)
                assert_close_dtype(out.float().cpu().numpy(), ref, dtype, atol32=1e-6 * (1 + _scale(ref)))


def test_partial_and_merge_through_the_c_abi_across_column_shards(oracle_mod):
    """Two column shards folded separately, states concatenated in shard order, merged: the path
    the multi-GPU split uses (ascending chunk, then ascending shard order)."""
    import torch

    import neptune_opt_b200._lib as L
    import neptune_opt_b200 as NB

    lib = L.load()
    gen = torch.Generator().manual_seed(5)
    for name in ("logsumexp", "stable_l2", "rmsnorm_max"):
        sk = NB.SKELETONS[name].id
        params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
        p = L.params_struct(params)
        x = (torch.randn(64, 50000, generator=gen) * 3).to(torch.bfloat16).cuda()
        shards = [(0, 20000), (20000, 30000)]
        chunk = 8192
        states = []
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for begin, width in shards:
            nparts = -(-width // chunk)
            st = torch.empty(64 * nparts * 4, dtype=torch.int32, device="cuda")
            rc = lib.nb200_fold_partial(sk, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 1, 64, 50000, begin,
                                        width, x.stride(0), 1, chunk, ctypes.c_void_p(st.data_ptr()), None, stream)
            L.check(rc, "partial")
            states.append(st.view(64, nparts, 4))
        allst = torch.cat(states, dim=1).contiguous()
        out = torch.empty(64, dtype=torch.bfloat16, device="cuda")
        rc = lib.nb200_fold_merge(sk, ctypes.byref(p), ctypes.c_void_p(allst.data_ptr()), 64, allst.shape[1],
                                  allst.shape[1], 1, ctypes.c_void_p(out.data_ptr()), 1, stream)
        L.check(rc, "merge")
        ref = oracle_mod.fold(name, _oracle_rows(x), params)
        assert_close_dtype(out.float().cpu().numpy(), ref, "bfloat16")


def test_softmax_and_log_softmax_match_oracle(oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(9)
    for dtype in DTYPES:
        for label, x in _inputs(dtype, gen):
            for log in (False, True):
                y, lse = NB.run_softmax_lse(x, log=log)
                assert y.shape == x.shape and y.dtype == x.dtype and y.is_contiguous()
                ry, rl = oracle_mod.softmax(_oracle_rows(x), log=log)
                got = y.float().reshape(ry.shape).cpu().numpy()
                if dtype == "float32":
                    assert_close_dtype(got, ry, dtype, rtol32=1e-5, atol32=1e-6 if log else 1e-37)
                else:
                    assert_close_dtype(got, ry, dtype, ulps=1, atol32=1e-6 if log else 1e-30)
                assert_close_dtype(lse.float().reshape(-1).cpu().numpy(), rl, dtype)
    sm = golden("softmax.npz")
    x = torch.from_numpy(sm["x"]).cuda()
    assert_close_dtype(NB.softmax(x).cpu().numpy(), sm["softmax"], "float32", atol32=1e-37)
    assert_close_dtype(NB.log_softmax(x).cpu().numpy(), sm["log_softmax"], "float32", atol32=1e-5)


def test_l2_normalize_matches_oracle(oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(13)
    for dtype in DTYPES:
        for label, x in _inputs(dtype, gen):
            y, norm = NB.run_l2_normalize(x)
            ry, rn = oracle_mod.l2_normalize(_oracle_rows(x), dtype)
            assert_close_dtype(y.float().reshape(ry.shape).cpu().numpy(), ry, dtype, atol32=1e-7)
            assert_close_dtype(norm.float().reshape(-1).cpu().numpy(), rn, dtype)


def test_rms_norm_matches_oracle_and_golden(oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(17)
    for dtype in DTYPES:
        dt = _t(dtype)
        for shape, plan in (((64, 4096), "serial"), ((33, 1000), "serial"), ((9, 1001), "serial"),
                            ((5, 32768), "serial"), ((3, 70000), "split"), ((2, 3, 768), "serial")):
            x = torch.randn(*shape, generator=gen).to(dt).cuda()
            gamma = (1 + 0.1 * torch.randn(shape[-1], generator=gen)).to(dt).cuda()
            before = x.clone()
            out = NB.run_rms_norm(x, gamma, eps=1e-6, plan=plan)
            assert out.is_contiguous() and out.dtype == dt and out.shape == x.shape
            assert torch.equal(x, before)
            ref = oracle_mod.rms_norm(_oracle_rows(x), gamma.float().cpu().numpy(), 1e-6, dtype)
            assert_rms_close(out.float().reshape(ref.shape).cpu().numpy(), ref, dtype)
        # strided gamma and transposed input
        x = torch.randn(512, 40, generator=gen).to(dt).cuda().t()
        g2 = (1 + 0.1 * torch.randn(1024, generator=gen)).to(dt).cuda()[::2]
        out = NB.run_rms_norm(x, g2)
        ref = oracle_mod.rms_norm(_oracle_rows(x), g2.float().cpu().numpy(), 1e-6, dtype)
        assert_rms_close(out.float().cpu().numpy(), ref, dtype)
    rms = golden("rms_norm.npz")
    for key in sorted({k.rsplit("|", 1)[0] for k in rms.files}):
        dtype = key.split("|")[0]
        x = torch.from_numpy(rms[key + "|x"]).to(_t(dtype)).cuda()
        g = torch.from_numpy(rms[key + "|gamma"]).to(_t(dtype)).cuda()
        assert_rms_close(NB.run_rms_norm(x, g).float().cpu().numpy(), rms[key + "|out"], dtype)


def test_host_row_rms_norm_streams_chunks_bit_exactly(oracle_mod):
    """nb200_rms_norm_host: rows in host memory, chunked through the device with overlapping copies,
    give bit for bit the device path's rows (and so the oracle's within the RMSNorm bound), for
    ragged last chunks, one-row chunks, pageable memory and the default chunking."""
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(23)
    cases = [((16384, 4096), torch.bfloat16, 0, True), ((1000, 768), torch.float16, 7, True),
             ((3, 2048), torch.float32, 1, False), ((5, 3, 1000), torch.bfloat16, 4, True),
             ((2, 512), torch.bfloat16, 4096, False)]
    for shape, dt, chunk, pinned in cases:
        x = torch.randn(*shape, generator=gen).to(dt)
        g = (1 + 0.1 * torch.randn(shape[-1], generator=gen)).to(dt)
        if pinned:
            x, g = x.pin_memory(), g.pin_memory()
        before = x.clone()
        out = NB.run_rms_norm_host(x, g, eps=1e-6, chunk_rows=chunk)
        torch.cuda.current_stream().synchronize()
        want = NB.run_rms_norm(x.cuda(), g.cuda(), eps=1e-6).cpu()
        assert out.shape == x.shape and out.dtype == dt and torch.equal(x, before)
        assert torch.equal(out, want), f"{shape} {dt} chunk_rows={chunk}"
    dtype = "float16"
    x = torch.randn(257, 1024, generator=gen).half().pin_memory()
    g = (1 + 0.1 * torch.randn(1024, generator=gen)).half().pin_memory()
    out = NB.run_rms_norm_host(x, g, eps=1e-6, chunk_rows=16)
    torch.cuda.current_stream().synchronize()
    ref = oracle_mod.rms_norm(x.float().numpy(), g.float().numpy(), 1e-6, dtype)
    assert_rms_close(out.float().numpy(), ref, dtype)


def test_segment_pool_bit_exact_on_reference_cases():
    import torch

    import neptune_opt_b200 as NB

    seg = golden("segment.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in seg.files})
    for key in keys:
        dtype, view, initial, reduce, kind = key.split("|")
        initial = None if initial == "None" else float(initial)
        data = torch.from_numpy(seg[key + "|data"]).to(_t(dtype)).cuda()
        segments = torch.from_numpy(seg[key + "|segments"]).cuda()
        if kind == "len" and view != "poisson":
            segments = segments.to(torch.int32)
        before = data.clone()
        out = NB.run_segment_pool(data, segments, reduce=reduce, initial=initial, offsets=(kind == "off"))
        got = out.float().cpu().numpy()
        ref = seg[key + "|out"]
        assert out.dtype == data.dtype and out.shape == ref.shape
        np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
        fin = ~np.isnan(ref)
        np.testing.assert_array_equal(got[fin], ref[fin])
        np.testing.assert_array_equal(np.signbit(got[fin]), np.signbit(ref[fin]))
        assert torch.equal(torch.nan_to_num(data, 7.0), torch.nan_to_num(before, 7.0))


def test_segment_pool_bit_exact_random_against_oracle(oracle_mod):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(21)
    for dtype in DTYPES:
        for channels in (128, 5, 300):
            lengths = torch.poisson(torch.full((700,), 20.0), generator=gen).clamp(0, 200).to(torch.int64)
            lengths[::97] = 0
            T = int(lengths.sum())
            data = torch.randn(T, channels, generator=gen).to(_t(dtype)).cuda()
            for reduce in ("sum", "mean"):
                for initial in (None, 0.5):
                    out = NB.run_segment_pool(data, lengths.cuda(), reduce=reduce, initial=initial)
                    spans, st = oracle_mod.segment_spans(lengths.numpy(), False, False, T)
                    ref = oracle_mod.segment_pool(data.float().cpu().numpy(), spans, reduce, initial, dtype)
                    got = out.float().cpu().numpy()
                    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
                    np.testing.assert_array_equal(got[~np.isnan(ref)], ref[~np.isnan(ref)])


def test_segment_spans_status_and_nan_for_invalid_descriptors(monkeypatch):
    import torch

    import neptune_opt_b200 as NB
    from neptune_opt_b200 import torch_op

    NB.segment_status()  # start from a clear word
    sp = golden("spans.npz")
    labels = sorted({k.rsplit("|", 1)[0] for k in sp.files})
    for label in labels:
        is_off, unsafe, nrows = (int(v) for v in sp[label + "|meta"])
        segs = torch.from_numpy(sp[label + "|segments"]).cuda()
        data = torch.zeros(nrows, 2, device="cuda")
        if is_off and segs.numel() == 0:
            continue
        out = NB.run_segment_pool(data, segs, offsets=bool(is_off), unsafe=bool(unsafe))
        status = NB.segment_status()
        error = str(sp[label + "|error"])
        if not error:
            assert status == 0, label
        else:
            with pytest.raises(RuntimeError) as info:
                torch_op.check_segment_status(status)
            assert str(info.value) in error, (label, str(info.value), error)
        assert out.shape[0] == (segs.numel() - 1 if is_off else segs.numel())
    monkeypatch.setenv("NEPTUNE_B200_SYNC_CHECKS", "1")
    with pytest.raises(RuntimeError, match="monotonic"):
        NB.run_segment_pool(torch.zeros(7, 2, device="cuda"), torch.tensor([0, 5, 3, 7], device="cuda"), offsets=True)
    assert NB.segment_status() == 0  # the failing check cleared the word
    # malformed spans pool to NaN without reading data; valid neighbours are unaffected
    monkeypatch.setenv("NEPTUNE_B200_SYNC_CHECKS", "0")
    for dtype in DTYPES:
        out = NB.run_segment_pool(torch.ones(7, 8, device="cuda", dtype=_t(dtype)),
                                  torch.tensor([0, 5, 3, 7], device="cuda"), offsets=True, reduce="sum")
        got = out.float().cpu().numpy()
        assert np.isnan(got[1]).all() and (got[0] == 5.0).all() and (got[2] == 4.0).all()
    assert NB.segment_status() == 8


def test_custom_ops_run_on_gpu_and_match_run():
    import torch

    import neptune_opt_b200 as NB

    x = torch.randn(17, 3000, device="cuda")
    h = NB.op_handle("lse_scaled", params={"T": 2.0, "tiny": 0.0}, keepdim=True)
    torch.testing.assert_close(h(x), NB.run("lse_scaled", x, keepdim=True, T=2.0), rtol=0, atol=0)
    torch.testing.assert_close(NB.logsumexp(x), torch.logsumexp(x, -1), rtol=1e-5, atol=1e-5)
    g = torch.randn(3000, device="cuda")
    rms = NB.state_op_handle("rms_norm", {"eps": 1e-6})
    torch.testing.assert_close(rms(x, g), NB.run_rms_norm(x, g), rtol=0, atol=0)
    sm = NB.softmax_op_handle(log=True)
    torch.testing.assert_close(sm(x), torch.log_softmax(x, -1), rtol=1e-5, atol=1e-5)
    seg = NB.segment_op_handle("segment_sum", {"initial": None, "offsets": True})
    data = torch.randn(10, 4, device="cuda")
    offs = torch.tensor([0, 3, 3, 10], device="cuda")
    torch.testing.assert_close(seg(data, offs), torch.segment_reduce(data, "sum", offsets=offs), rtol=0, atol=0)


def test_launches_are_counted_by_the_library():
    import torch

    import neptune_opt_b200 as NB

    before = NB.launch_count()
    NB.run("logsumexp", torch.randn(4, 100, device="cuda"))
    NB.run_rms_norm(torch.randn(4, 100, device="cuda"), torch.randn(100, device="cuda"))
    assert NB.launch_count() - before == 2


def test_streaming_kernels_never_timed_out():
    """Every bounded wait of the bulk-copy kernels completed in this process."""
    import torch

    import neptune_opt_b200._lib as L

    torch.cuda.synchronize()
    assert L.stream_fault() == 0


def test_bulk_copy_paths_match_oracle(oracle_mod):
    """The bulk-copy ring kernels: AUTO sends contiguous rows of 8-32 KB there (fold, softmax, L2,
    RMSNorm), and an explicit STREAM launch forces them for 1-8 KB rows and for split-plan chunks."""
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200._lib as L

    lib = L.load()
    gen = torch.Generator().manual_seed(17)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for dtype, ncols in (("float32", 4096), ("bfloat16", 12288), ("float16", 6000)):
        x = (torch.randn(96, ncols, generator=gen) * 2).to(_t(dtype)).cuda()
        rows = _oracle_rows(x)
        for name in ("logsumexp", "stable_l2", "variance"):
            params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
            ref = oracle_mod.fold(name, rows, params)
            assert_close_dtype(NB.run(name, x, **params).float().cpu().numpy(), ref, dtype,
                               atol32=1e-6 * (1 + _scale(ref)))
        y, lse = NB.run_softmax_lse(x)
        ry, rl = oracle_mod.softmax(rows)
        assert_close_dtype(y.float().cpu().numpy(), ry, dtype)
        assert_close_dtype(lse.float().cpu().numpy(), rl, dtype)
        g = (1 + 0.1 * torch.randn(ncols, generator=gen)).to(_t(dtype)).cuda()
        assert_rms_close(NB.run_rms_norm(x, g, eps=1e-6).float().cpu().numpy(),
                         oracle_mod.rms_norm(rows, g.float().cpu().numpy(), 1e-6, dtype), dtype)

    forced = L.launch_struct(L.VARIANT_STREAM, 0, 0, 0)
    p = L.params_struct({"tiny": 0.0})
    for dtype, shape in (("float32", (50, 2048)), ("bfloat16", (40, 1024))):
        x = (torch.randn(*shape, generator=gen) * 3).to(_t(dtype)).cuda()
        ref = oracle_mod.fold("logsumexp", _oracle_rows(x), {"tiny": 0.0})
        out = torch.empty(shape[0], dtype=x.dtype, device="cuda")
        L.check(lib.nb200_fold(0, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), DTYPES.index(dtype), shape[0],
                               shape[1], shape[1], 1, ctypes.c_void_p(out.data_ptr()), ctypes.byref(forced), stream),
                "stream fold")
        assert_close_dtype(out.float().cpu().numpy(), ref, dtype, atol32=1e-6 * (1 + _scale(ref)))
    x = (torch.randn(16, 70000, generator=gen) * 3).to(torch.bfloat16).cuda()
    ref = oracle_mod.fold("logsumexp", _oracle_rows(x), {"tiny": 0.0})
    nparts = -(-70000 // 8192)
    scratch = torch.empty(int(lib.nb200_fold_split_scratch_bytes(16, nparts)), dtype=torch.uint8, device="cuda")
    out = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    L.check(lib.nb200_fold_split(0, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 1, 16, 70000, 70000, 1, 8192,
                                 ctypes.c_void_p(scratch.data_ptr()), scratch.numel(), ctypes.c_void_p(out.data_ptr()),
                                 ctypes.byref(forced), stream), "stream split")
    assert_close_dtype(out.float().cpu().numpy(), ref, "bfloat16")


def test_long_length_vectors_build_spans_bit_exactly(oracle_mod):
    """Length vectors past 16384 segments take the three-launch, many-CTA span construction: the
    spans and the status bits must equal the oracle's for valid vectors, strided int32 views, and
    violations placed in interior blocks (negative length, oversized length, lengths that do not
    cover the rows with and without `unsafe`)."""
    import torch

    import neptune_opt_b200._lib as L

    lib = L.load()
    gen = torch.Generator().manual_seed(23)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def run(lengths, nrows, unsafe, idt):
        n = lengths.shape[0]
        spans = torch.full((n + 1,), -7, dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        L.check(lib.nb200_segment_spans(ctypes.c_void_p(lengths.data_ptr()), idt, n, lengths.stride(0), int(unsafe),
                                        nrows, ctypes.c_void_p(spans.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                                        stream), "spans")
        torch.cuda.synchronize()
        return spans.cpu().numpy(), int(status.item())

    for nseg in (16385, 100000, 200000, 4096 * 37 + 1):
        lengths = torch.poisson(torch.full((nseg,), 20.0), generator=gen).clamp(1, 200).to(torch.int64)
        T = int(lengths.sum())
        cases = [("valid", lengths.clone(), T, False)]
        bad = lengths.clone()
        bad[nseg // 2] = -3
        cases.append(("negative", bad, T, False))
        big = lengths.clone()
        big[nseg - 5] = T + 10
        cases.append(("oversized", big, T, False))
        cases.append(("short cover", lengths.clone(), T + 5, False))
        cases.append(("short cover, unsafe", lengths.clone(), T + 5, True))
        for label, lens, nrows, unsafe in cases:
            want, wst = oracle_mod.segment_spans(lens.numpy(), False, unsafe, nrows)
            got, gst = run(lens.cuda(), nrows, unsafe, L.INDEX_CODES["int64"])
            assert np.array_equal(got, want) and gst == wst, f"{nseg} {label}: status {gst} vs {wst}"
        wide = torch.zeros(nseg, 2, dtype=torch.int32)
        wide[:, 0] = lengths.to(torch.int32)
        view = wide.cuda()[:, 0]  # int32, element stride 2
        want, wst = oracle_mod.segment_spans(lengths.numpy(), False, False, T)
        got, gst = run(view, T, False, L.INDEX_CODES["int32"])
        assert np.array_equal(got, want) and gst == wst, f"{nseg} strided int32"


def test_cluster_rows_fold_matches_oracle(oracle_mod):
    """Few, very wide rows: one thread-block cluster per row, CTA states merged through distributed
    shared memory. AUTO takes it for up to 296 rows wider than 32 KB; an explicit cluster launch forces
    2, 8 or 16 CTAs per row; nonfinite rows keep the log family's status semantics; rows the
    cluster kernel cannot take (strided) are refused by an explicit launch and folded by AUTO."""
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200._lib as L

    lib = L.load()
    gen = torch.Generator().manual_seed(53)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def launch(name, params, x, csize):
        p = L.params_struct(params)
        out = torch.full((x.shape[0],), float("nan"), dtype=x.dtype, device="cuda")
        forced = L.launch_struct(L.VARIANT_CLUSTER, 0, 0, csize)
        rc = lib.nb200_fold(NB.SKELETONS[name].id, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()),
                            DTYPES.index(str(x.dtype)[6:]), x.shape[0], x.shape[1], x.stride(0), 1,
                            ctypes.c_void_p(out.data_ptr()), ctypes.byref(forced), stream)
        return rc, out

    names = ("logsumexp", "lse_biased", "lse_scaled", "softcap_lse", "stable_l2", "linear_attn", "decay_renorm",
             "sumsq_div", "rmsnorm_max")
    for dtype in DTYPES:
        for shape in ((1, 262144), (3, 70000), (8, 65536), (74, 40000)):
            x = (torch.randn(*shape, generator=gen) * 3).to(_t(dtype)).cuda()
            rows = _oracle_rows(x)
            for name in names:
                params = {**NB.param_defaults(name), **TEST_PARAMS.get(name, {})}
                ref = oracle_mod.fold(name, rows, params)
                atol = max(1e-6 * (1 + _scale(ref)), _sum_floor(name, rows, params))
                assert_close_dtype(NB.run(name, x, **params).float().cpu().numpy(), ref, dtype, atol32=atol)
                if shape[0] <= 8 and name in ("logsumexp", "stable_l2", "rmsnorm_max"):
                    for csize in (2, 8, 16):
                        rc, out = launch(name, params, x, csize)
                        L.check(rc, f"cluster fold {csize}")
                        assert_close_dtype(out.float().cpu().numpy(), ref, dtype, atol32=atol)
    # nonfinite rows: the reference's log-family status (NaN wins, then +inf, -inf rows)
    special = golden("fold.npz")["logsumexp|0|special|float32|x"]
    wide = np.full((special.shape[0], 50000), -np.inf, np.float32)
    wide[:, :special.shape[1]] = special
    wide[:, 40000] = 0.5
    wide[[1, 4], 40000] = -np.inf
    for dtype in DTYPES:
        x = torch.from_numpy(wide).to(_t(dtype)).cuda()
        ref = oracle_mod.fold("logsumexp", x.float().cpu().numpy(), {"tiny": 0.0})
        rc, out = launch("logsumexp", {"tiny": 0.0}, x, 8)
        L.check(rc, "cluster fold special")
        assert_nonfinite_equal(out.float().cpu().numpy(), ref)
        assert_close_dtype(out.float().cpu().numpy(), ref, dtype)
    # strided rows: refused by an explicit cluster launch, folded by AUTO's other paths
    base = (torch.randn(4, 2 * 40000 + 2, generator=gen)).cuda()
    x = base[:, 1:80001:2]
    p = L.params_struct({"tiny": 0.0})
    out = torch.empty(4, device="cuda")
    forced = L.launch_struct(L.VARIANT_CLUSTER, 0, 0, 0)
    rc = lib.nb200_fold(0, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 0, 4, 40000, x.stride(0), x.stride(1),
                        ctypes.c_void_p(out.data_ptr()), ctypes.byref(forced), stream)
    assert rc == L.NB200_ERR_ARG
    assert_close_dtype(NB.run("logsumexp", x).cpu().numpy(), oracle_mod.fold("logsumexp", _oracle_rows(x), {}),
                       "float32")


def test_cluster_rows_rms_norm_matches_oracle(oracle_mod):
    """RMSNorm of few, very wide rows through one cluster per row (the partial sums of squares meet
    in every CTA's shared memory), and the fallback when a row exceeds the cluster's registers."""
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200._lib as L

    lib = L.load()
    gen = torch.Generator().manual_seed(59)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for dtype in DTYPES:
        dt = _t(dtype)
        for shape in ((1, 65536), (2, 131072), (7, 40000), (64, 16384 + 8)):
            x = torch.randn(*shape, generator=gen).to(dt).cuda()
            g = (1 + 0.1 * torch.randn(shape[1], generator=gen)).to(dt).cuda()
            ref = oracle_mod.rms_norm(_oracle_rows(x), g.float().cpu().numpy(), 1e-6, dtype)
            assert_rms_close(NB.run_rms_norm(x, g, eps=1e-6, plan="split").float().cpu().numpy(), ref, dtype)
            for csize in (2, 16):
                y = torch.full_like(x, float("nan"))
                forced = L.launch_struct(L.VARIANT_CLUSTER, 0, 0, csize)
                rc = lib.nb200_rms_norm(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(g.data_ptr()),
                                        DTYPES.index(dtype), shape[0], shape[1], shape[1], 1, 1, ctypes.c_double(1e-6),
                                        ctypes.c_void_p(y.data_ptr()), ctypes.byref(forced), stream)
                nvec = shape[1] * x.element_size() // 16
                if -(-nvec // csize) > 256 * 8:
                    # more vectors per CTA than its registers hold: refused, nothing written
                    torch.cuda.synchronize()
                    assert rc == L.NB200_ERR_ARG and torch.isnan(y).all()
                    continue
                L.check(rc, f"cluster rms {csize}")
                assert_rms_close(y.float().cpu().numpy(), ref, dtype)
    # wider than 16 CTAs x 256 threads x 8 vectors: AUTO falls back to the one-CTA-per-row kernel
    x = torch.randn(1, 16 * 256 * 8 * 4 + 4, generator=gen).cuda()
    g = torch.ones(x.shape[1], device="cuda")
    ref = oracle_mod.rms_norm(_oracle_rows(x), g.float().cpu().numpy(), 1e-6, "float32")
    assert_rms_close(NB.run_rms_norm(x, g, eps=1e-6, plan="split").float().cpu().numpy(), ref, "float32")
