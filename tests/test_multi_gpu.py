"""Multi-GPU run of the column-sharded split plan (the one multi-GPU path with an exchange), on
every GPU of the box up to 8.

Each rank folds its column shard of a bf16 [64, 100000] block into chunk states; they move either
through one NCCL all-gather or through NVLink peer memory (PeerExchange: epoch-tagged stores into
every rank's buffer, a merge that reads each state until it carries the call's epoch -- the fold storing into the buffers
itself, or a partial fold plus push and merge kernels, alternating call by call), and every rank merges them in
ascending (rank, chunk) order. Both must equal, bit for bit, the single-GPU merge of the same states in the
same order, match the oracle within 1 bf16 ulp, agree with each other on inputs that change from
call to call, and replay from a captured CUDA graph. Runs as one spawned process per GPU; skipped
with fewer than two GPUs.
"""
from __future__ import annotations

import ctypes
import os
import socket

import pytest

from conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

ROWS, NCOLS, CHUNK = 64, 100000, 8192


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    import datetime

    import torch
    import torch.distributed as td

    from neptune_opt_b200 import _lib
    from neptune_opt_b200.parallel import PeerExchange, shard_rows, sharded_split_fold

    # NVLS off: no NVLink multicast object is created for the collectives (the exchange uses none)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                          device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator().manual_seed(21)
        x = (torch.randn(ROWS, NCOLS, generator=gen) * 3).to(torch.bfloat16)
        c0, c1 = shard_rows(NCOLS, world, rank)  # contiguous column block of this rank
        shard = x[:, c0:c1].contiguous().cuda()
        out = sharded_split_fold("logsumexp", shard, NCOLS, params={"tiny": 0.0}, chunk=CHUNK)
        widths = [shard_rows(NCOLS, world, r)[1] - shard_rows(NCOLS, world, r)[0] for r in range(world)]
        again = sharded_split_fold("logsumexp", shard, NCOLS, params={"tiny": 0.0}, chunk=CHUNK, widths=widths)
        # the same through NVLink peer memory: every call equals the all-gather path bit for bit,
        # with inputs that change from call to call (a stale epoch or parity would show), then
        # captured in a CUDA graph and replayed
        ex = PeerExchange(ROWS, max(-(-w // CHUNK) for w in widths))
        try:
            peer_ok = []
            for i in range(6):
                # alternate the fused form and the partial + push + merge form: same protocol
                xi = shard * (1.0 + 0.25 * i)
                want = sharded_split_fold("logsumexp", xi, NCOLS, params={"tiny": 0.0}, chunk=CHUNK, widths=widths)
                got = sharded_split_fold("logsumexp", xi, NCOLS, params={"tiny": 0.0}, chunk=CHUNK, widths=widths,
                                         exchange=ex, fused=(i % 2 == 0))
                peer_ok.append(bool(torch.equal(want, got)))
            first = sharded_split_fold("logsumexp", shard, NCOLS, params={"tiny": 0.0}, chunk=CHUNK, widths=widths,
                                       exchange=ex)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                with torch.cuda.graph(graph):
                    replayed = sharded_split_fold("logsumexp", shard, NCOLS, params={"tiny": 0.0}, chunk=CHUNK,
                                                  widths=widths, exchange=ex)
            graph_ok = []
            for _ in range(3):
                graph.replay()
                torch.cuda.synchronize()
                graph_ok.append(bool(torch.equal(replayed, out)))
            del graph
            faults = ctypes.c_uint32(0)
            _lib.check(_lib.load().nb200_stream_fault(ctypes.byref(faults)), "fault word")
        finally:
            ex.close()
        torch.cuda.synchronize()
        if rank == 0:
            torch.save({"out": out.cpu(), "again": again.cpu(), "peer": first.cpu(), "peer_ok": peer_ok,
                        "graph_ok": graph_ok, "faults": int(faults.value)}, result_path)
        td.barrier()
    finally:
        td.destroy_process_group()


def test_sharded_split_over_nccl_matches_single_gpu(tmp_path, oracle_mod):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 8)  # every GPU of the box, up to the exchange's 8 ranks
    result = str(tmp_path / "r0.pt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = torch.load(result)

    from conftest import assert_close_dtype
    from neptune_opt_b200.parallel import _cuda_merge, _cuda_partial, shard_rows

    gen = torch.Generator().manual_seed(21)
    x = (torch.randn(ROWS, NCOLS, generator=gen) * 3).to(torch.bfloat16)
    states = []
    for r in range(world):  # the same shards and chunking on one GPU, states in (rank, chunk) order
        c0, c1 = shard_rows(NCOLS, world, r)
        states.append(_cuda_partial("logsumexp", {"tiny": 0.0}, x[:, c0:c1].contiguous().cuda(), c0, NCOLS, CHUNK))
    width = max(s.shape[1] for s in states)
    for i, s in enumerate(states):
        if s.shape[1] < width:
            pad = torch.zeros(ROWS, width - s.shape[1], 4, dtype=s.dtype, device=s.device)
            pad[..., 0] = torch.tensor(float("-inf")).view(torch.int32)
            states[i] = torch.cat([s, pad], dim=1)
    merged = _cuda_merge("logsumexp", {"tiny": 0.0}, torch.cat(states, dim=1).contiguous(),
                         torch.empty(ROWS, dtype=torch.bfloat16, device="cuda"))
    assert torch.equal(got["out"], merged.cpu()) and torch.equal(got["again"], merged.cpu())
    assert torch.equal(got["peer"], merged.cpu()), "peer-memory exchange differs from the merged states"
    assert all(got["peer_ok"]), f"peer exchange differs from the all-gather path on calls {got['peer_ok']}"
    assert all(got["graph_ok"]), f"graph replays of the peer exchange differ: {got['graph_ok']}"
    assert got["faults"] == 0, f"fault word {got['faults']:#x}"
    ref = oracle_mod.fold("logsumexp", x.float().numpy(), {"tiny": 0.0})
    assert_close_dtype(got["out"].float().numpy(), ref, "bfloat16")
