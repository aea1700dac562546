"""Parity at every benchmark configuration at its full size, on the inputs bench.py builds.

Each test builds the configuration with bench.py's own workload builder (same seeds, same device
generator, same launches), runs one bench step and compares the step's output with the CPU oracle
over the whole batch. Bars (the reference-equivalence contract):
  * fp32 softmax / logsumexp: rtol 1e-5 (atol 1e-37 for softmax values that underflow);
  * bf16 / fp16 results: within 1 ulp of the oracle's fp32 value before narrowing;
  * RMSNorm bf16: every element equals the reference's two roundings (x*scale to bf16, then the
    gamma product to bf16, emitters.py:576-595) applied to an intermediate x*scale within 1 bf16
    ulp of the oracle's; the count of elements that differ from the oracle at all is reported and
    bounded (a last-bit difference of the fp32 scale, from the summation order of sum x^2, moves
    the first rounding);
  * ordered segment pooling: bit-exact, sum and mean, 200000 segments.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close_dtype, cuda_available, round_to, ulp_of

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


@pytest.fixture(scope="module")
def bench_mod():
    import bench

    return bench


@pytest.fixture(scope="module")
def nb():
    import neptune_opt_b200 as NB

    NB.load()
    return NB


def _run_step0(torch, r):
    r["step"](0)
    torch.cuda.synchronize()
    return r["io0"]


def test_softmax_logsumexp_fp32_8192x2048_full(bench_mod, nb, oracle_mod):
    import torch

    r = bench_mod.make_softmax(torch, nb, 2000)
    io = _run_step0(torch, r)
    x = io["x"].cpu().numpy()
    assert (x[::64, 0] == 80.0).all()
    ry, rl = oracle_mod.softmax(x)
    assert_close_dtype(io["lse"].cpu().numpy(), rl, "float32", rtol32=1e-5)
    assert_close_dtype(io["y"].cpu().numpy(), ry, "float32", rtol32=1e-5, atol32=1e-37)
    del r, io
    r = bench_mod.make_lse(torch, nb, 2000)
    io = _run_step0(torch, r)
    ref = oracle_mod.fold("logsumexp", io["x"].cpu().numpy(), {"tiny": 0.0})
    assert_close_dtype(io["out"].cpu().numpy(), ref, "float32", rtol32=1e-5)
    torch.cuda.empty_cache()


def test_rms_norm_bf16_16384x4096_full(bench_mod, nb, oracle_mod):
    import torch

    r = bench_mod.make_rms(torch, nb, 1000)
    io = _run_step0(torch, r)
    x = io["x"].float().cpu().numpy()
    gamma = io["gamma"].float().cpu().numpy()
    got = io["y"].float().cpu().numpy()
    del r, io
    torch.cuda.empty_cache()
    want = oracle_mod.rms_norm(x, gamma, 1e-6, "bfloat16")
    scale = oracle_mod.rms_scale(x, 1e-6)
    # the reference's stages on the oracle's scale: a = bf16(x * scale), y = bf16(a * gamma)
    a = round_to(x * scale[:, None], "bfloat16")
    assert np.array_equal(round_to(a * gamma[None, :], "bfloat16"), want)
    diff = got != want
    n_diff = int(diff.sum())
    if n_diff:
        # every differing element is the reference's rounding of a neighbouring intermediate:
        # y == bf16(a' * gamma) with a' one bf16 ulp above or below a
        rows, cols = np.nonzero(diff)
        # the two bf16 neighbours of a: its bit pattern +-1 is one ulp larger / smaller in magnitude
        bits = torch.from_numpy(np.ascontiguousarray(a[rows, cols])).to(torch.bfloat16).view(torch.int16)
        g = gamma[cols]
        gv = got[rows, cols]
        explained = np.zeros(rows.shape, bool)
        for delta in (1, -1):
            nb_a = (bits + delta).view(torch.bfloat16).float().numpy()
            explained |= gv == round_to(nb_a * g, "bfloat16")
        assert explained.all(), f"{int((~explained).sum())} elements not explained by a one-ulp intermediate"
    beyond_1ulp = int((np.abs(got.astype(np.float64) - want) > ulp_of(want, "bfloat16")).sum())
    print(f"\nrms_norm bf16 [16384,4096]: {n_diff} of {got.size} elements differ from the oracle, "
          f"{beyond_1ulp} by more than 1 ulp")
    assert n_diff <= 1e-4 * got.size


def test_l2_normalize_fp16_65536x768_full(bench_mod, nb, oracle_mod):
    import torch

    r = bench_mod.make_l2(torch, nb, 2000)
    io = _run_step0(torch, r)
    x = io["x"].float().cpu().numpy()
    ry, rn = oracle_mod.l2_normalize(x, "float32")
    assert_close_dtype(io["y"].float().cpu().numpy(), ry, "float16")
    assert_close_dtype(io["norm"].float().cpu().numpy(), rn, "float16")
    del r, io
    torch.cuda.empty_cache()


def test_split_plan_logsumexp_bf16_512x262144_full(bench_mod, nb, oracle_mod):
    import torch

    r = bench_mod.make_wide_lse(torch, nb, 2000)
    io = _run_step0(torch, r)
    x = io["x"].float().cpu().numpy()
    got = io["out"].float().cpu().numpy()
    del r, io
    torch.cuda.empty_cache()
    ref = oracle_mod.fold("logsumexp", x, {"tiny": 0.0}, block=16384)
    assert_close_dtype(got, ref, "bfloat16", ulps=1)


@pytest.mark.parametrize("reduce", ["sum", "mean"])
def test_segment_pool_fp16_200000_segments_full(bench_mod, nb, oracle_mod, reduce):
    import torch

    r = bench_mod.make_segments(torch, nb, 2000, reduce)
    assert r["T"] == 3997578
    io = _run_step0(torch, r)
    got = io["last"]["out"].float().cpu().numpy()
    data = io["data"].float().cpu().numpy()
    lengths = io["lengths"].numpy()
    offsets = io["offsets"].cpu().numpy()
    del r, io
    torch.cuda.empty_cache()
    spans, status = oracle_mod.segment_spans(lengths, False, False, data.shape[0])
    assert status == 0 and np.array_equal(spans, offsets)
    want = oracle_mod.segment_pool(data, spans, reduce, None, "float16")
    assert got.shape == (200000, 128)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got, want) and np.array_equal(np.signbit(got), np.signbit(want))
