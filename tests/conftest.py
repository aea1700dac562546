"""Shared fixtures and tolerance helpers.

`-m "not gpu"` runs the oracle against the reference's golden vectors, the host-side contracts and
the C ABI's loading/exports (no GPU work). `-m gpu` runs the CUDA kernels through the C ABI and
compares them with the oracle (tests/../oracle) and the golden vectors.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


TORCH_DTYPES = ("float32", "bfloat16", "float16")


def torch_dtype(name: str):
    import torch

    return getattr(torch, name)


def round_to(values, dtype: str) -> np.ndarray:
    """RTNE narrowing of fp32 values to `dtype`, back as fp32 (torch's conversion)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(np.asarray(values, np.float32)))
    return t.to(torch_dtype(dtype)).float().numpy()


def ulp_of(values, dtype: str) -> np.ndarray:
    """Spacing of `dtype` at each value (1 ulp), as fp32."""
    mant = {"float32": 23, "bfloat16": 7, "float16": 10}[dtype]
    emin = {"float32": -126, "bfloat16": -126, "float16": -14}[dtype]
    v = np.abs(np.asarray(values, np.float64))
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(v > 0, v, 1.0)))
    e = np.maximum(e, emin)
    return np.ldexp(1.0, (e - mant).astype(np.int64))


def assert_nonfinite_equal(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    assert np.array_equal(np.isnan(got), np.isnan(ref)), "NaN positions differ"
    inf = np.isinf(ref)
    assert np.array_equal(np.isinf(got), inf), "inf positions differ"
    assert np.array_equal(got[inf], ref[inf]), "inf signs differ"


def assert_close_dtype(got, ref32, dtype: str, *, rtol32: float = 1e-5, atol32: float = 0.0, ulps: float = 1.0):
    """The parity bar: fp32 within rtol32 (+atol32); bf16/fp16 within `ulps` of the dtype after the
    fp32 compute (ref32 is the fp32 oracle value before narrowing). Nonfinite values must match."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref32, np.float64)
    # A finite fp32 value can overflow when narrowed (e.g. 1e5 in fp16): nonfinite positions are
    # those of the narrowed reference.
    narrowed = ref if dtype == "float32" else round_to(ref32, dtype).astype(np.float64)
    assert_nonfinite_equal(got, narrowed)
    fin = np.isfinite(narrowed)
    g, r = got[fin], ref[fin]
    if dtype == "float32":
        err = np.abs(g - r)
        bound = rtol32 * np.abs(r) + atol32
        bad = err > bound
        assert not bad.any(), f"fp32 mismatch: max err {err.max():.3e}, worst rel {(err / np.maximum(np.abs(r), 1e-30)).max():.3e}"
    else:
        err = np.abs(g - r)
        bound = ulps * ulp_of(r, dtype) + atol32
        bad = err > bound
        assert not bad.any(), f"{dtype} mismatch beyond {ulps} ulp at {np.argwhere(bad)[:5].tolist()}: " \
                              f"got {g[bad][:5]}, ref {r[bad][:5]}"


def assert_rms_close(got, ref, dtype: str):
    """RMSNorm bar: the contract rounds twice (x * scale to the input dtype, then the gamma product),
    so a last-bit difference of the fp32 scale (summation order of sum x^2) can move the first
    rounding by one ulp and the result by up to two. fp32: rtol 1e-5. bf16/fp16: every element
    within 2 ulp and all but 0.1% within 1 ulp of the reference value."""
    if dtype == "float32":
        assert_close_dtype(got, ref, "float32", rtol32=1e-5, atol32=1e-6)
        return
    assert_close_dtype(got, ref, dtype, ulps=2)
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    fin = np.isfinite(ref)
    over = np.abs(got[fin] - ref[fin]) > ulp_of(ref[fin], dtype)
    assert over.mean() <= 1e-3, f"{over.mean():.2e} of elements beyond 1 ulp"


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.lib()
    return oracle


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False
