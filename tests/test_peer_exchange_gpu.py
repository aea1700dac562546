"""The peer-memory exchange of the column-sharded split plan on one GPU, through the C ABI.

Two exchange buffers on the same device stand in for two ranks' buffers, so the kernels' own
checks run without a second GPU:
* world = 1: push + merge, and the fused nb200_peer_fold (fold storing into the buffers, then the
  merge), equal nb200_fold_merge of the same states, bit for bit, call after call (mixing forms);
* a rank that never pushes: the merge's bounded wait for its states runs out after about a second,
  fault bit 2 (0x4) is reported once, and the merge writes the rows as NaN -- after the push
  kernel and after the fused form;
* a buffer initialised for another layout: the push stores nothing into it and the merge reads
  nothing from it (fault bit 3, 0x8).
No GPU is faulted or hung: the wait is bounded by the kernel and ends with a status the host reads.
"""
from __future__ import annotations

import ctypes

import pytest

from conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

ROWS, CHUNK = 64, 4096


def _buffer(lib, rows, world, nparts):
    import torch

    nbytes = int(lib.nb200_peer_buffer_bytes(rows, world, nparts))
    storage = torch.zeros(nbytes + 256, dtype=torch.uint8, device="cuda")
    pad = (-storage.data_ptr()) % 256
    return storage, storage[pad:pad + nbytes]


def _states(lib, L, x, nparts):
    import torch

    import neptune_opt_b200 as NB

    rows, width = x.shape
    st = torch.empty(rows, nparts, 4, dtype=torch.int32, device="cuda")
    p = L.params_struct({"tiny": 0.0})
    L.check(lib.nb200_fold_partial(NB.SKELETONS["logsumexp"].id, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 0,
                                   rows, width, 0, width, x.stride(0), 1, CHUNK, ctypes.c_void_p(st.data_ptr()), None,
                                   _stream()), "partial")
    return st


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _init(lib, L, buf, rows, world, nparts):
    L.check(lib.nb200_peer_init(ctypes.c_void_p(buf.data_ptr()), rows, world, nparts, _stream()), "peer init")


def _push(lib, states, rows, nparts, bufs, rank, own):
    peers = (ctypes.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])
    return lib.nb200_peer_push(ctypes.c_void_p(states.data_ptr()), rows, states.shape[1], nparts, peers, len(bufs),
                               rank, ctypes.c_void_p(own.data_ptr()), _stream())


def _merge(lib, L, buf, rows, nparts, world, out):
    import neptune_opt_b200 as NB

    p = L.params_struct({"tiny": 0.0})
    return lib.nb200_peer_merge(NB.SKELETONS["logsumexp"].id, ctypes.byref(p), ctypes.c_void_p(buf.data_ptr()), rows,
                                nparts, world, ctypes.c_void_p(out.data_ptr()), 0, _stream())


@pytest.mark.parametrize("rows,nparts", [(ROWS, 3), (512, 4)])
def test_single_rank_exchange_equals_the_merge_kernel(rows, nparts):
    """192 chunk items: the 4 warps of a CTA share each item; 2048: one warp per item. The fused
    form must decompose the items as the partial fold does in both cases."""
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200._lib as L

    lib = L.load()
    torch.cuda.synchronize()
    L.stream_fault()
    gen = torch.Generator().manual_seed(41)
    x = (torch.randn(rows, nparts * CHUNK, generator=gen) * 3).cuda()
    states = _states(lib, L, x, nparts)
    _keep, buf = _buffer(lib, rows, 1, nparts)
    _init(lib, L, buf, rows, 1, nparts)
    want = torch.empty(rows, device="cuda")
    p = L.params_struct({"tiny": 0.0})
    L.check(lib.nb200_fold_merge(NB.SKELETONS["logsumexp"].id, ctypes.byref(p), ctypes.c_void_p(states.data_ptr()),
                                 rows, nparts, nparts, 1, ctypes.c_void_p(want.data_ptr()), 0, _stream()), "merge")
    for i in range(6):  # consecutive calls walk the epochs and parities, alternating the two forms
        out = torch.full((rows,), float("nan"), device="cuda")
        if i % 2:
            L.check(_fold(lib, L, x, nparts, [buf], 0, buf, out), "peer fold")
        else:
            L.check(_push(lib, states, rows, nparts, [buf], 0, buf), "push")
            L.check(_merge(lib, L, buf, rows, nparts, 1, out), "peer merge")
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"call {i}"
    assert L.stream_fault() == 0


def test_fused_form_refuses_chunks_held_as_resident_rows():
    """Chunks of 4 KB or less are folded by the partial fold as resident rows, a decomposition the
    fused form does not have: it refuses them before launching anything."""
    import torch

    import neptune_opt_b200 as NB
    import neptune_opt_b200._lib as L
    from neptune_opt_b200.parallel import PeerExchange

    lib = L.load()
    torch.cuda.synchronize()
    L.stream_fault()
    x = torch.randn(ROWS, 4 * 1024, device="cuda")
    _keep, buf = _buffer(lib, ROWS, 1, 4)
    _init(lib, L, buf, ROWS, 1, 4)
    out = torch.zeros(ROWS, device="cuda")
    p = L.params_struct({"tiny": 0.0})
    before = NB.launch_count()
    rc = lib.nb200_peer_fold(NB.SKELETONS["logsumexp"].id, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 0, ROWS,
                             x.shape[1], x.shape[1], x.stride(0), 1024, 4,
                             (ctypes.c_void_p * 1)(buf.data_ptr()), 1, 0, ctypes.c_void_p(buf.data_ptr()),
                             ctypes.c_void_p(out.data_ptr()), _stream())
    torch.cuda.synchronize()
    assert rc == L.NB200_ERR_UNSUPPORTED and "push form" in L.last_error()
    assert NB.launch_count() == before and int(out.count_nonzero()) == 0 and L.stream_fault() == 0
    assert not PeerExchange.fold_eligible(x, 1024) and PeerExchange.fold_eligible(x, 2048)


def _fold(lib, L, x, nparts, bufs, rank, own, out):
    import neptune_opt_b200 as NB

    p = L.params_struct({"tiny": 0.0})
    peers = (ctypes.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])
    rows, width = x.shape
    return lib.nb200_peer_fold(NB.SKELETONS["logsumexp"].id, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 0, rows,
                               width, width, x.stride(0), CHUNK, nparts, peers, len(bufs), rank,
                               ctypes.c_void_p(own.data_ptr()), ctypes.c_void_p(out.data_ptr()), _stream())


def test_merge_wait_runs_out_when_a_rank_never_pushes():
    import torch

    import neptune_opt_b200._lib as L

    lib = L.load()
    torch.cuda.synchronize()
    L.stream_fault()
    gen = torch.Generator().manual_seed(43)
    x = (torch.randn(ROWS, 2 * CHUNK, generator=gen) * 3).cuda()
    nparts = 2
    states = _states(lib, L, x, nparts)
    keep0, buf0 = _buffer(lib, ROWS, 2, nparts)
    keep1, buf1 = _buffer(lib, ROWS, 2, nparts)
    for b in (buf0, buf1):
        _init(lib, L, b, ROWS, 2, nparts)
    out = torch.zeros(ROWS, device="cuda")  # the merge writes NaN rows
    L.check(_push(lib, states, ROWS, nparts, [buf0, buf1], 0, buf0), "push")  # "rank 1" never pushes
    L.check(_merge(lib, L, buf0, ROWS, nparts, 2, out), "peer merge")
    torch.cuda.synchronize()
    assert L.stream_fault() & 0x4, "the merge's wait for the missing rank's states did not report running out"
    assert torch.isnan(out).all(), "the merge did not write NaN rows although a rank's states never arrived"
    assert L.stream_fault() == 0, "the fault word was not cleared by reading it"
    # the fused form: its merge's wait for "rank 1" runs out the same way
    for b in (buf0, buf1):
        _init(lib, L, b, ROWS, 2, nparts)
    out = torch.zeros(ROWS, device="cuda")  # the merge writes NaN rows
    L.check(_fold(lib, L, x, nparts, [buf0, buf1], 0, buf0, out), "peer fold")
    torch.cuda.synchronize()
    assert L.stream_fault() & 0x4, "the fused form's wait did not report running out"
    assert torch.isnan(out).all()
    assert L.stream_fault() == 0


def test_layout_mismatch_stores_and_reads_nothing():
    import torch

    import neptune_opt_b200._lib as L

    lib = L.load()
    torch.cuda.synchronize()
    L.stream_fault()
    gen = torch.Generator().manual_seed(47)
    x = (torch.randn(ROWS, 2 * CHUNK, generator=gen) * 3).cuda()
    nparts = 2
    states = _states(lib, L, x, nparts)
    keep0, buf0 = _buffer(lib, ROWS, 2, nparts)
    keep1, buf1 = _buffer(lib, ROWS, 2, nparts)
    _init(lib, L, buf0, ROWS, 2, nparts)
    _init(lib, L, buf1, ROWS // 2, 2, nparts)  # initialised for another layout
    torch.cuda.synchronize()
    buf1[256:].fill_(0x5A)
    before = buf1.clone()
    L.check(_push(lib, states, ROWS, nparts, [buf0, buf1], 0, buf0), "push")
    torch.cuda.synchronize()
    assert L.stream_fault() & 0x8, "the push did not report the destination's layout mismatch"
    assert torch.equal(buf1, before), "the push stored into a buffer of another layout"
    out = torch.zeros(ROWS, device="cuda")  # the merge writes NaN rows
    L.check(_merge(lib, L, buf1, ROWS, nparts, 2, out), "peer merge")
    torch.cuda.synchronize()
    assert L.stream_fault() & 0x8 and torch.isnan(out).all()
    # a buffer that was never initialised is refused the same way
    keep2, buf2 = _buffer(lib, ROWS, 1, nparts)
    L.check(_push(lib, states, ROWS, nparts, [buf2], 0, buf2), "push")
    torch.cuda.synchronize()
    assert L.stream_fault() & 0x8
    assert int(buf2.count_nonzero()) == 0
