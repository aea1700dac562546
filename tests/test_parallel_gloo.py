"""Multi-rank host logic on CPU: world-size-2 gloo process groups.

The CUDA kernels do not run here; the per-shard fold and the merge are supplied by the oracle, so
these tests check what the multi-GPU path adds -- sharding arithmetic, the one all-gather of chunk
states, the ascending (rank, chunk) merge order and the segment partition that keeps every segment
on one rank -- against the single-process answer.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from neptune_opt_b200 import parallel


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, fn, *args):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(r, world, port, q, fn, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, ok, payload = q.get(timeout=180)
        results[rank] = (ok, payload)
    for p in procs:
        p.join(timeout=60)
    for rank, (ok, payload) in sorted(results.items()):
        assert ok, f"rank {rank}: {payload}"
    return [results[r][1] for r in range(world)]


def _entry(rank, world, port, q, fn, args):
    import sys
    import traceback

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as td

    td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, True, fn(rank, world, *args)))
    except Exception:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))
    finally:
        td.destroy_process_group()


def _split_worker(rank, world, name, params, rows, ncols, chunk, uneven):
    import oracle

    rng = np.random.default_rng(42)
    x = (rng.standard_normal((rows, ncols)) * 3).astype(np.float32)
    if uneven:
        cuts = [0, ncols // 3, ncols]
    else:
        cuts = [parallel.shard_rows(ncols, world, r)[0] for r in range(world)] + [ncols]
    lo, hi = cuts[rank], cuts[rank + 1]

    def partial_fn(nm, prm, x_shard, col_begin, ncols_total, ch):
        st = oracle.partial(nm, x, prm, col_begin, x_shard.shape[1], ch)  # reads only the shard
        return torch.from_numpy(st.view(np.int32).reshape(rows, -1, 4).copy())

    def merge_fn(nm, prm, states, out):
        st = states.contiguous().numpy().view(oracle.STATE_DTYPE).reshape(rows, -1)
        out.copy_(torch.from_numpy(oracle.merge(nm, st, prm)))
        return out

    shard = torch.from_numpy(x[:, lo:hi].copy())
    out = parallel.sharded_split_fold(name, shard, ncols, params=params, chunk=chunk,
                                      partial_fn=partial_fn, merge_fn=merge_fn)
    serial = oracle.merge(name, oracle.partial(name, x, params, 0, ncols, chunk), params)
    # the same chunk grouping, merged in one process in ascending (shard, chunk) order
    same = np.concatenate([oracle.partial(name, x, params, cuts[r], cuts[r + 1] - cuts[r], chunk)
                           for r in range(world)], axis=1)
    return out.numpy(), serial, oracle.merge(name, same, params)


@pytest.mark.parametrize("name,params", [("logsumexp", {"tiny": 0.0}), ("stable_l2", {}),
                                         ("rmsnorm_max", {"eps": 1e-6}), ("lse_scaled", {"T": 2.0, "tiny": 0.0})])
@pytest.mark.parametrize("uneven", [False, True])
def test_sharded_split_fold_matches_single_process(name, params, uneven):
    outs = _run(2, _split_worker, name, params, 16, 5000, 1024, uneven)
    for out, serial, same_order in outs:
        np.testing.assert_array_equal(out, same_order)  # exchange preserves the certified order
        np.testing.assert_allclose(out, serial, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(outs[0][0], outs[1][0])


def _exchange_worker(rank, world, rows, ncols, chunk):
    """sharded_split_fold's exchange branch with a stand-in for PeerExchange that moves the states
    with gloo: the local states, padded to the slot width, must merge to the all-gather result."""
    import oracle
    import torch.distributed as td

    rng = np.random.default_rng(5)
    x = (rng.standard_normal((rows, ncols)) * 3).astype(np.float32)
    cuts = [0, ncols // 3, ncols]
    lo, hi = cuts[rank], cuts[rank + 1]
    widths = [cuts[r + 1] - cuts[r] for r in range(world)]
    nparts = max(-(-w // chunk) for w in widths)

    def partial_fn(nm, prm, x_shard, col_begin, ncols_total, ch):
        st = oracle.partial(nm, x, prm, col_begin, x_shard.shape[1], ch)
        return torch.from_numpy(st.view(np.int32).reshape(rows, -1, 4).copy())

    def merge_fn(nm, prm, states, out):
        st = states.contiguous().numpy().view(oracle.STATE_DTYPE).reshape(rows, -1)
        out.copy_(torch.from_numpy(oracle.merge(nm, st, prm)))
        return out

    class GlooExchange:
        def __init__(self, parts):
            self.world, self.nparts, self.calls = world, parts, 0

        def exchange_and_merge(self, name, params, states, out):
            self.calls += 1
            pad = torch.zeros(rows, self.nparts - states.shape[1], 4, dtype=torch.int32)
            pad[..., 0] = torch.tensor(float("-inf")).view(torch.int32)
            mine = torch.cat([states, pad], dim=1)
            every = [torch.empty_like(mine) for _ in range(world)]
            td.all_gather(every, mine)
            return merge_fn(name, params, torch.cat(every, dim=1), out)

    shard = torch.from_numpy(x[:, lo:hi].copy())
    kw = dict(params={"tiny": 0.0}, chunk=chunk, partial_fn=partial_fn, merge_fn=merge_fn, widths=widths)
    ref = parallel.sharded_split_fold("logsumexp", shard, ncols, **kw)
    ex = GlooExchange(nparts)
    got = parallel.sharded_split_fold("logsumexp", shard, ncols, exchange=ex, **kw)
    refused = False
    try:
        parallel.sharded_split_fold("logsumexp", shard, ncols, exchange=GlooExchange(nparts + 1), **kw)
    except ValueError:
        refused = True
    return ref.numpy(), got.numpy(), ex.calls, refused


def test_sharded_split_fold_exchange_branch_matches_all_gather():
    for ref, got, calls, refused in _run(2, _exchange_worker, 8, 3000, 512):
        np.testing.assert_array_equal(ref, got)
        assert calls == 1 and refused


def _peer_setup_worker(rank, world):
    """PeerExchange set-up that fails locally (no GPU here): every rank must raise, none may hang."""
    try:
        parallel.PeerExchange(8, 2, device="cuda:0")
    except RuntimeError as exc:
        return "raised", str(exc)
    return "constructed", ""


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the failure path of a machine without GPUs")
def test_peer_exchange_setup_failure_raises_on_every_rank():
    for outcome, message in _run(2, _peer_setup_worker):
        assert outcome == "raised" and "set-up failed" in message
        assert "rank 0" in message and "rank 1" in message  # each rank reports every rank's failure


def _segment_worker(rank, world, T, nseg, channels):
    import oracle

    gen = torch.Generator().manual_seed(3)
    lengths = torch.poisson(torch.full((nseg,), 20.0), generator=gen).clamp(1, 200).to(torch.int64)
    lengths[-1] += T - int(lengths.sum()) if int(lengths.sum()) < T else 0
    offsets = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)])
    data = torch.randn(int(offsets[-1]), channels, generator=gen).to(torch.float16).float().numpy()
    sh = parallel.shard_segments(offsets, world, rank)
    local = parallel.local_offsets(offsets, sh)
    part = oracle.segment_pool(data[sh.row_begin:sh.row_end], local.numpy(), "mean", None, "float16")
    gathered = [None] * world
    import torch.distributed as td

    td.all_gather_object(gathered, (sh.seg_begin, sh.seg_end, sh.row_end - sh.row_begin, part))
    full = oracle.segment_pool(data, offsets.numpy(), "mean", None, "float16")
    return gathered, full, int(offsets[-1])


def test_segment_shards_are_whole_balanced_and_bit_exact():
    results = _run(2, _segment_worker, 4000, 200, 16)
    gathered, full, total = results[0]
    assert gathered[0][0] == 0 and gathered[-1][1] == 200
    assert gathered[0][1] == gathered[1][0]  # contiguous, no segment split across ranks
    assert abs(gathered[0][2] - total / 2) <= 200  # balanced to within one segment
    stitched = np.concatenate([g[3] for g in gathered], axis=0)
    np.testing.assert_array_equal(stitched, full)


def test_shard_rows_and_heads_cover_exactly():
    for rows in (0, 1, 7, 16384):
        for world in (1, 2, 3, 8):
            blocks = [parallel.shard_rows(rows, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == rows
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in blocks) - min(b - a for a, b in blocks) <= 1
    assert parallel.shard_heads(8, 32, 8, 7) == (224, 256)
    with pytest.raises(ValueError):
        parallel.shard_rows(4, 2, 2)


def test_segment_shard_edge_cases():
    off = torch.tensor([0, 0, 0, 5, 5, 9])
    shards = [parallel.shard_segments(off, 3, r) for r in range(3)]
    assert shards[0].seg_begin == 0 and shards[-1].seg_end == 5
    assert all(shards[i].seg_end == shards[i + 1].seg_begin for i in range(2))
    assert sum(s.row_end - s.row_begin for s in shards) == 9
    one = parallel.shard_segments(torch.tensor([0]), 2, 1)
    assert one.seg_begin == one.seg_end == 0


def test_fused_exchange_eligibility_follows_the_partial_folds_layout_rules():
    """The fused form takes contiguous, 16-byte aligned shards in chunks wider than 4 KB; narrower
    chunks (which the partial fold holds as resident rows), strided shards and unaligned widths go
    to the partial fold + push form."""
    import torch

    from neptune_opt_b200.parallel import PeerExchange

    f32 = torch.empty(64, 8192)
    bf16 = torch.empty(64, 8192, dtype=torch.bfloat16)
    assert PeerExchange.fold_eligible(f32, 2048) and not PeerExchange.fold_eligible(f32, 1024)
    assert PeerExchange.fold_eligible(bf16, 4096) and not PeerExchange.fold_eligible(bf16, 2048)
    assert not PeerExchange.fold_eligible(f32[:, ::2], 2048)        # strided columns
    assert not PeerExchange.fold_eligible(f32[:, 1:4097], 2048)     # unaligned start
    assert not PeerExchange.fold_eligible(torch.empty(64, 8190), 2048)  # width not a multiple of 16 B
