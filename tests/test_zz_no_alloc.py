"""The split plan's no-allocation entry point, through the C ABI.

nb200_fold_split_noalloc is for callers that cannot allocate device memory (a host that only hands
over input and output buffers, a fixed device-memory budget, a path where an allocation call would
synchronise). It keeps the chunk states in a fixed array inside the library instead of caller
scratch. These checks compare it with the allocating entry point, nb200_fold_split, on two calls in
a row with different shapes -- the second call must not see the first call's leftover states -- and
check that an oversized request is refused. This file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import pytest

from conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

DTYPE_CODE = {"float32": 0, "bfloat16": 1, "float16": 2}


def _split(lib, L, sk, params, x, chunk, out, noalloc, stream):
    import torch

    rows, ncols = x.shape
    p = L.params_struct(params)
    if noalloc:
        return lib.nb200_fold_split_noalloc(sk, ctypes.byref(p), x.data_ptr(), DTYPE_CODE[str(x.dtype)[6:]], rows,
                                            ncols, x.stride(0), x.stride(1), chunk, out.data_ptr(), stream)
    nparts = -(-ncols // chunk)
    scratch = torch.empty(int(lib.nb200_fold_split_scratch_bytes(rows, nparts)), dtype=torch.uint8, device=x.device)
    return lib.nb200_fold_split(sk, ctypes.byref(p), x.data_ptr(), DTYPE_CODE[str(x.dtype)[6:]], rows, ncols,
                                x.stride(0), x.stride(1), chunk, scratch.data_ptr(), scratch.numel(), out.data_ptr(),
                                None, stream)


def test_no_alloc_split_matches_the_allocating_entry_point_on_two_calls():
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200._lib as L

    lib = L.load()
    gen = torch.Generator().manual_seed(31)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = [  # (skeleton, params, rows, ncols, chunk, dtype)
        ("logsumexp", {"tiny": 0.0}, 256, 65536, 16384, torch.bfloat16),
        ("stable_l2", {}, 48, 50000, 4096, torch.float32),
    ]
    for name, params, rows, ncols, chunk, dtype in cases:
        x = (torch.randn(rows, ncols, generator=gen) * 3).to(dtype).cuda()
        want = torch.empty(rows, dtype=dtype, device="cuda")
        got = torch.full((rows,), float("nan"), dtype=dtype, device="cuda")
        sk = NB.SKELETONS[name].id
        L.check(_split(lib, L, sk, params, x, chunk, want, False, stream), "nb200_fold_split")
        L.check(_split(lib, L, sk, params, x, chunk, got, True, stream), "nb200_fold_split_noalloc")
        torch.cuda.synchronize()
        # the same kernels fold the same chunks in the same order: the results are identical bit for bit
        assert torch.equal(got, want), f"{name}: no-alloc split differs from nb200_fold_split"


def test_no_alloc_split_refuses_requests_beyond_its_scratch():
    import torch

    import neptune_opt_b200._lib as L

    lib = L.load()
    x = torch.zeros(65537, 64, device="cuda")  # sized for the request, though it is refused unread
    out = torch.empty(65537, device="cuda")
    p = L.params_struct({"tiny": 0.0})
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # 65537 rows x 4 chunks = 262148 chunk states > 262144: refused before any launch (x is never read)
    rc = lib.nb200_fold_split_noalloc(0, ctypes.byref(p), x.data_ptr(), 0, 65537, 64, 64, 1, 16, out.data_ptr(),
                                      stream)
    assert rc == L.NB200_ERR_CAPACITY
    assert "262144" in L.last_error()
