"""The C ABI library loads, exports every symbol include/*.h declares, and rejects bad arguments
before touching the GPU (these calls never reach a CUDA API, so they run without a device)."""
from __future__ import annotations

import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT


def _declared_symbols() -> set:
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(nb200_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    import neptune_opt_b200._lib as L

    lib = L.load()
    declared = _declared_symbols()
    assert len(declared) >= 14
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"
    assert "sm_100a" in lib.nb200_version().decode()


def test_library_is_in_tree_and_built_for_sm100a():
    import neptune_opt_b200._lib as L

    assert os.path.dirname(L.LIB_PATH) == os.path.join(ROOT, "neptune_opt_b200")
    data = open(L.LIB_PATH, "rb").read()
    assert b"sm_100a" in data or b"compute_100a" in data


def test_argument_validation_happens_before_any_launch():
    import neptune_opt_b200._lib as L

    lib = L.load()
    p = L.params_struct({"tiny": 0.0})
    null = ctypes.c_void_p(0)
    # bad dtype, bad width, bad skeleton, bad parameter domain -> NB200_ERR_ARG, no CUDA call
    assert lib.nb200_fold(0, ctypes.byref(p), null, 7, 4, 8, 8, 1, null, None, null) == L.NB200_ERR_ARG
    assert "dtype" in L.last_error()
    assert lib.nb200_fold(0, ctypes.byref(p), null, 0, 4, 0, 0, 1, null, None, null) == L.NB200_ERR_ARG
    assert "width" in L.last_error()
    assert lib.nb200_fold(99, ctypes.byref(p), null, 0, 4, 8, 8, 1, null, None, null) == L.NB200_ERR_ARG
    bad = L.params_struct({"T": -1.0})
    assert lib.nb200_fold(2, ctypes.byref(bad), null, 0, 4, 8, 8, 1, null, None, null) == L.NB200_ERR_ARG
    assert "'T'" in L.last_error()
    # zero rows is a successful no-op
    assert lib.nb200_fold(0, ctypes.byref(p), null, 0, 0, 8, 8, 1, null, None, null) == L.NB200_OK
    # split capacity and two-pass refusal
    assert lib.nb200_fold_split(0, ctypes.byref(p), null, 0, 0, 4097, 4097, 1, 1, null, 0, null, None, null) \
        == L.NB200_ERR_CAPACITY
    assert "capacity" in L.last_error()
    assert lib.nb200_fold_split(9, ctypes.byref(p), null, 0, 0, 8, 8, 1, 4, null, 0, null, None, null) \
        == L.NB200_ERR_UNSUPPORTED
    assert lib.nb200_fold_split_scratch_bytes(3, 5) == 3 * 5 * 16
    # RMSNorm eps and launch policy checks
    assert lib.nb200_rms_norm(null, null, 1, 2, 8, 8, 1, 1, 0.0, null, None, null) == L.NB200_ERR_ARG
    bad_launch = L.launch_struct(L.VARIANT_CTA_ROW, 48, 0)
    assert lib.nb200_fold(0, ctypes.byref(p), null, 0, 1, 8, 8, 1, null, ctypes.byref(bad_launch), null) \
        == L.NB200_ERR_ARG
    # segments: index dtype and reduce mode
    assert lib.nb200_segment_spans(null, 5, 1, 1, 0, 1, null, null, null) == L.NB200_ERR_ARG
    assert lib.nb200_segment_pool(null, 0, 1, 1, 1, 1, null, 1, 1, 1, 7, 0, 0, null, null, null) == L.NB200_ERR_ARG
    assert lib.nb200_segment_pool(null, 0, 1, 1, 1, 1, null, 9, 1, 1, 0, 0, 0, null, null, null) == L.NB200_ERR_ARG
    assert lib.nb200_segment_pool(null, 0, 1, 4, 4, 1, null, 1, 1, 0, 0, 0, 0, null, null, null) == L.NB200_OK
    # attention: shape, head_dim, scale and alignment are refused on the host (the pointers are
    # never dereferenced); an empty problem is a successful no-op
    fake = ctypes.c_void_p(1 << 20)
    assert lib.nb200_attention(null, null, null, null, None, 1, 1, 0, 128, 0, 0.1, null) == L.NB200_OK
    assert lib.nb200_attention(null, fake, fake, fake, None, 1, 1, 8, 128, 0, 0.1, null) == L.NB200_ERR_ARG
    assert lib.nb200_attention(fake, fake, fake, fake, None, 1, 1, 8, 64, 0, 0.1, null) == L.NB200_ERR_UNSUPPORTED
    assert "head_dim" in L.last_error()
    assert lib.nb200_attention(fake, fake, fake, fake, None, 1, 1, 8, 128, 0, -1.0, null) == L.NB200_ERR_ARG
    odd = ctypes.c_void_p((1 << 20) + 2)
    assert lib.nb200_attention(odd, fake, fake, fake, None, 1, 1, 8, 128, 1, 0.1, null) == L.NB200_ERR_ARG
    assert "aligned" in L.last_error()
    # host-row RMSNorm: workspace size, then dtype / size / eps / pointer / workspace checks on
    # the host (before any CUDA call); zero rows is a successful no-op
    need = lib.nb200_rms_norm_host_work_bytes(1, 4096, 2048)
    assert need == 8192 + 4 * 2048 * 8192
    assert lib.nb200_rms_norm_host_work_bytes(1, 4096, 0) == 8192 + 4 * (16 << 20)
    assert lib.nb200_rms_norm_host_work_bytes(7, 4096, 0) == -1
    assert lib.nb200_rms_norm_host(fake, fake, 7, 4, 8, 1e-6, fake, 0, fake, need, null) == L.NB200_ERR_ARG
    assert lib.nb200_rms_norm_host(fake, fake, 1, 4, 0, 1e-6, fake, 0, fake, need, null) == L.NB200_ERR_ARG
    assert lib.nb200_rms_norm_host(fake, fake, 1, 4, 8, 0.0, fake, 0, fake, need, null) == L.NB200_ERR_ARG
    assert lib.nb200_rms_norm_host(null, fake, 1, 4, 8, 1e-6, fake, 0, fake, need, null) == L.NB200_ERR_ARG
    assert lib.nb200_rms_norm_host(fake, fake, 1, 4, 8, 1e-6, fake, 2, odd, need, null) == L.NB200_ERR_ARG
    assert "aligned" in L.last_error()
    small = lib.nb200_rms_norm_host_work_bytes(1, 8, 2) - 1
    assert lib.nb200_rms_norm_host(fake, fake, 1, 4, 8, 1e-6, fake, 2, fake, small, null) == L.NB200_ERR_ARG
    assert lib.nb200_rms_norm_host(null, null, 1, 0, 8, 1e-6, null, 0, null, 0, null) == L.NB200_OK


def test_check_maps_status_to_reference_exceptions():
    import neptune_opt_b200._lib as L

    L.load()
    with pytest.raises(ValueError):
        L.check(L.NB200_ERR_ARG, "x")
    with pytest.raises(NotImplementedError):
        L.check(L.NB200_ERR_CAPACITY, "x")
    with pytest.raises(RuntimeError):
        L.check(L.NB200_ERR_LAUNCH, "x")
    L.check(L.NB200_OK, "x")


def test_product_path_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "neptune_opt_b200")
    for path in glob.glob(os.path.join(pkg, "**", "*.py"), recursive=True):
        text = open(path).read()
        assert not re.search(r"^\s*(import|from)\s+oracle\b", text, flags=re.M), path
