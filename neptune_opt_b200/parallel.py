"""Multi-GPU partitioning of the fused reductions: one process per GPU, torch.distributed plumbing.

The reference has no multi-GPU path (its roadmap declares it out of scope). Here every region
partitions into independent units, so ranks need no data-path collective:

* row-last folds, softmax, L2-normalize, RMSNorm: contiguous blocks of rows (`shard_rows`);
* ordered segment pooling: contiguous blocks of whole segments, cut where the token counts balance
  (`shard_segments`); each segment stays on one rank, so the storage-dtype rounding order -- and
  with it the bit-exact result -- is unchanged;
* attention: blocks of (batch, head) pairs (`shard_heads`).

The one exchange is the split plan for ultra-wide rows when the reduction axis itself is sharded
across GPUs (`sharded_split_fold`): each rank folds its column shard into per-row chunk states
(16 bytes each) and every rank merges all of them in ascending (rank, chunk) order -- the same
certified order as the single-GPU split plan. The states move either through one all-gather or,
with a `PeerExchange`, through NVLink peer memory: the folding (or pushing) kernel stores them into
every rank's buffer, each state tagged with the call's epoch inside its 16 bytes, and the merging
kernel reads each state until it carries that epoch (no collective, no flag, no host step).
"""
from __future__ import annotations

import ctypes
import dataclasses


def shard_rows(rows: int, world: int, rank: int) -> tuple:
    """[begin, end) of rank's contiguous row block; blocks differ in size by at most one row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(rows, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_heads(batch: int, heads: int, world: int, rank: int) -> tuple:
    """[begin, end) over the flattened batch*heads pairs."""
    return shard_rows(batch * heads, world, rank)


@dataclasses.dataclass(frozen=True)
class SegmentShard:
    seg_begin: int       # first segment of this rank
    seg_end: int         # one past the last segment
    row_begin: int       # first data row those segments read
    row_end: int         # one past the last data row


def shard_segments(offsets, world: int, rank: int) -> SegmentShard:
    """Contiguous segments whose token ranges split the data rows evenly.

    `offsets` is the CSR boundary array (length nsegments + 1, nondecreasing, host or device). The
    cut before rank r is the first segment boundary at or after r * T / world, so every rank gets
    whole segments and about T / world rows.
    """
    import torch

    off = torch.as_tensor(offsets).to("cpu", torch.int64)
    nseg = off.numel() - 1
    if nseg < 0:
        raise ValueError("offsets needs at least one boundary")
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    first, last = int(off[0]), int(off[-1])
    total = last - first

    def cut(r):
        if r <= 0:
            return 0
        if r >= world:
            return nseg
        target = first + (total * r + world - 1) // world
        return int(torch.searchsorted(off[:-1].contiguous(), torch.tensor(target), right=False))

    s0, s1 = cut(rank), cut(rank + 1)
    s1 = max(s0, s1)
    return SegmentShard(s0, s1, int(off[s0]), int(off[s1]))


def local_offsets(offsets, shard: SegmentShard):
    """The rank's offsets rebased to its own data rows (first entry 0)."""
    import torch

    off = torch.as_tensor(offsets)
    return off[shard.seg_begin:shard.seg_end + 1] - off[shard.seg_begin]


# ---------------------------------------------------------------- the sharded split plan
def _cuda_partial(name, params, x_shard, col_begin, ncols_total, chunk):
    """Chunk states [rows, nparts] (as int32 [rows, nparts, 4]) of a column shard, via the C ABI."""
    import torch

    from neptune_opt_b200 import _lib
    from neptune_opt_b200.skeletons import SKELETONS, checked_params
    from neptune_opt_b200.template import _on_device, current_stream, dtype_code

    rows, width = x_shard.shape
    nparts = -(-width // chunk)
    states = torch.empty(rows, nparts, 4, dtype=torch.int32, device=x_shard.device)
    p = _lib.params_struct(checked_params(name, params))
    lib = _lib.load()
    with _on_device(x_shard.device):
        rc = lib.nb200_fold_partial(SKELETONS[name].id, ctypes.byref(p), ctypes.c_void_p(x_shard.data_ptr()),
                                    dtype_code(x_shard.dtype), rows, ncols_total, 0, width, x_shard.stride(0),
                                    x_shard.stride(1), chunk, ctypes.c_void_p(states.data_ptr()), None,
                                    ctypes.c_void_p(current_stream(x_shard.device)))
    _lib.check(rc, f"neptune {name} partial")
    return states


def _cuda_merge(name, params, states, out):
    """Merge [rows, nparts, 4] states in ascending part order into out[rows] via the C ABI."""
    from neptune_opt_b200 import _lib
    from neptune_opt_b200.skeletons import SKELETONS, checked_params
    from neptune_opt_b200.template import _on_device, current_stream, dtype_code

    rows, nparts = states.shape[0], states.shape[1]
    p = _lib.params_struct(checked_params(name, params))
    lib = _lib.load()
    with _on_device(states.device):
        rc = lib.nb200_fold_merge(SKELETONS[name].id, ctypes.byref(p), ctypes.c_void_p(states.data_ptr()), rows,
                                  nparts, states.stride(0) // 4, states.stride(1) // 4,
                                  ctypes.c_void_p(out.data_ptr()), dtype_code(out.dtype),
                                  ctypes.c_void_p(current_stream(states.device)))
    _lib.check(rc, f"neptune {name} merge")
    return out


class PeerExchange:
    """Exchange buffers of the column-sharded split plan, mapped across the ranks of `group`.

    Every rank allocates one buffer of `nb200_peer_buffer_bytes(rows, world, nparts)` bytes on its
    GPU, records the layout in it (`nb200_peer_init`) and maps the others' with CUDA IPC (handles
    swapped once with all_gather_object). A `sharded_split_fold(..., exchange=ex)` call then moves
    the chunk states with two kernels -- epoch-tagged stores into every peer's buffer, and a merge
    that reads each state until it carries the call's epoch -- instead of a collective. `nparts` is the per-rank slot width: the
    largest number of chunks any rank's shard has. Create it on every rank of the group (it
    synchronises them) and `close()` it on every rank.

    Faults: the merge's wait for the ranks' states is bounded (about a second); when it runs out
    (a rank did not push) the kernel sets bit 2 of `nb200_stream_fault` and writes those rows as
    NaN, and a call whose layout differs from a buffer's sets bit 3 and stores nothing (a merge on
    such a buffer writes every row as NaN).
    Nothing on the host notices by itself: pass `check=True` to `sharded_split_fold` (it
    synchronises and raises), or read `neptune_opt_b200._lib.stream_fault()`. After either fault
    the ranks' epochs disagree, so this exchange refuses further calls: close it on every rank and
    build a new one.
    """

    def __init__(self, rows: int, nparts: int, group=None, device=None):
        import torch
        import torch.distributed as td

        from neptune_opt_b200 import _lib

        self.group = group
        self.world = td.get_world_size(group)
        self.rank = td.get_rank(group)
        self.rows, self.nparts = int(rows), int(nparts)
        self._lib = lib = _lib.load()
        self._opened, self.peers = [], None
        self.faulted = False
        nbytes = int(lib.nb200_peer_buffer_bytes(self.rows, self.world, self.nparts))
        if nbytes < 0:
            raise ValueError(f"no peer exchange for rows={rows}, world={self.world}, nparts={nparts} (world <= 8)")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        # Every collective below runs on every rank whatever happened locally, and every decision is
        # taken from gathered results, so a failure on one rank raises on all of them together.
        mine = None
        try:
            self._storage = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
            pad = (-self._storage.data_ptr()) % 256
            self.buffer = self._storage[pad:pad + nbytes]
            with torch.cuda.device(device):
                _lib.check(lib.nb200_peer_init(ctypes.c_void_p(self.buffer.data_ptr()), self.rows, self.world,
                                               self.nparts, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                           "peer exchange init")
            handle = (ctypes.c_char * 64)()
            offset = ctypes.c_int64()
            _lib.check(lib.nb200_ipc_handle(ctypes.c_void_p(self.buffer.data_ptr()), handle, ctypes.byref(offset)),
                       "peer exchange handle")
            torch.cuda.synchronize(device)  # the layout is recorded before any peer can write into it
            mine = (bytes(handle), int(offset.value), self.rows, self.nparts)
        except Exception as exc:  # noqa: BLE001 -- reported on every rank below
            mine = ("error", f"rank {self.rank}: {exc}")
        everyone = [None] * self.world
        td.all_gather_object(everyone, mine, group=group)
        errors = [e[1] for e in everyone if e[0] == "error"]
        if errors:
            raise RuntimeError("peer exchange set-up failed: " + "; ".join(errors))
        # Every rank writes into every other rank's buffer at offsets computed from (rows, nparts):
        # the layouts must agree before anything is mapped.
        layouts = {(rows_r, parts_r) for _, _, rows_r, parts_r in everyone}
        if len(layouts) != 1:
            raise ValueError(f"ranks disagree on the exchange layout (rows, nparts): {sorted(layouts)}")
        ptrs, failure = [], None
        for r, (h, off, _, _) in enumerate(everyone):
            if r == self.rank:
                ptrs.append(self.buffer.data_ptr())
                continue
            base = ctypes.c_void_p()
            if lib.nb200_ipc_open(h, ctypes.byref(base)) != 0:
                failure = f"rank {self.rank} cannot map rank {r}: {_lib.last_error()}"
                break
            self._opened.append(base.value)
            ptrs.append(base.value + off)
        failures = [None] * self.world
        td.all_gather_object(failures, failure, group=group)
        failures = [f for f in failures if f]
        if failures:
            for base in self._opened:
                lib.nb200_ipc_close(ctypes.c_void_p(base))
            self._opened = []
            raise RuntimeError("peer exchange mapping failed: " + "; ".join(failures))
        td.barrier(group=group)  # every rank has mapped every buffer before the first push
        self.peers = (ctypes.c_void_p * self.world)(*ptrs)

    def exchange_and_merge(self, name, params, states, out):
        """Push this rank's states [rows, nlocal, 4] and merge all ranks' into out[rows]."""
        from neptune_opt_b200 import _lib
        from neptune_opt_b200.skeletons import SKELETONS, checked_params
        from neptune_opt_b200.template import _on_device, current_stream, dtype_code

        import torch

        if self.peers is None:
            raise RuntimeError("the peer exchange is closed")
        if self.faulted:
            raise RuntimeError("the peer exchange faulted (a bounded wait ran out or a layout differed); "
                               "close it on every rank and set up a new one")
        if states.dtype != torch.int32 or states.dim() != 3 or states.shape[2] != 4 or not states.is_contiguous():
            raise ValueError("states must be a contiguous int32 [rows, nlocal, 4] tensor of chunk states")
        rows, nlocal = states.shape[0], states.shape[1]
        if rows != self.rows or nlocal > self.nparts:
            raise ValueError(f"states [{rows}, {nlocal}] do not fit the exchange ({self.rows} rows, "
                             f"{self.nparts} parts per rank)")
        if out.dim() != 1 or out.numel() != rows or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [{rows}] tensor")
        if states.device != self.buffer.device or out.device != self.buffer.device:
            raise ValueError(f"states and out must be on the exchange's device {self.buffer.device}")
        p = _lib.params_struct(checked_params(name, params))
        lib = self._lib
        with _on_device(states.device):
            stream = ctypes.c_void_p(current_stream(states.device))
            _lib.check(lib.nb200_peer_push(ctypes.c_void_p(states.data_ptr()), rows, nlocal, self.nparts,
                                           self.peers, self.world, self.rank,
                                           ctypes.c_void_p(self.buffer.data_ptr()), stream), "peer push")
            _lib.check(lib.nb200_peer_merge(SKELETONS[name].id, ctypes.byref(p),
                                            ctypes.c_void_p(self.buffer.data_ptr()), rows, self.nparts,
                                            self.world, ctypes.c_void_p(out.data_ptr()), dtype_code(out.dtype),
                                            stream), "peer merge")
        return out

    def fold(self, name, params, x_shard, ncols_total, chunk, out):
        """The whole call in two launches (nb200_peer_fold): fold this rank's contiguous shard
        x_shard [rows, width] in `chunk`-column chunks storing the states straight into every rank's
        buffer, tagged with the call's epoch), then wait for everyone's and merge into out[rows].
        Same result, bit for bit, as the partial fold followed by `exchange_and_merge`."""
        from neptune_opt_b200 import _lib
        from neptune_opt_b200.skeletons import SKELETONS, checked_params
        from neptune_opt_b200.template import _on_device, current_stream, dtype_code

        if self.peers is None:
            raise RuntimeError("the peer exchange is closed")
        if self.faulted:
            raise RuntimeError("the peer exchange faulted (a bounded wait ran out or a layout differed); "
                               "close it on every rank and set up a new one")
        rows, width = x_shard.shape
        if rows != self.rows or -(-width // chunk) > self.nparts:
            raise ValueError(f"shard [{rows}, {width}] in {chunk}-column chunks does not fit the exchange "
                             f"({self.rows} rows, {self.nparts} parts per rank)")
        if out.dim() != 1 or out.numel() != rows or not out.is_contiguous() or out.dtype != x_shard.dtype:
            raise ValueError(f"out must be a contiguous [{rows}] tensor of the shard's dtype")
        if x_shard.device != self.buffer.device or out.device != self.buffer.device:
            raise ValueError(f"x_shard and out must be on the exchange's device {self.buffer.device}")
        p = _lib.params_struct(checked_params(name, params))
        with _on_device(x_shard.device):
            _lib.check(self._lib.nb200_peer_fold(SKELETONS[name].id, ctypes.byref(p),
                                                 ctypes.c_void_p(x_shard.data_ptr()), dtype_code(x_shard.dtype), rows,
                                                 int(ncols_total), width, x_shard.stride(0), int(chunk), self.nparts,
                                                 self.peers, self.world, self.rank,
                                                 ctypes.c_void_p(self.buffer.data_ptr()),
                                                 ctypes.c_void_p(out.data_ptr()),
                                                 ctypes.c_void_p(current_stream(x_shard.device))), "peer fold")
        return out

    @staticmethod
    def fold_eligible(x_shard, chunk) -> bool:
        """Whether a shard can take the fused form (`fold`): contiguous 16-byte aligned rows whose
        width, stride and chunk are multiples of 16 bytes, in chunks wider than 4 KB (narrower ones
        the partial fold holds as resident rows, which the fused form does not)."""
        es = x_shard.element_size()
        return (x_shard.dim() == 2 and x_shard.stride(1) == 1 and x_shard.data_ptr() % 16 == 0
                and (x_shard.shape[0] <= 1 or (x_shard.stride(0) * es) % 16 == 0)
                and (x_shard.shape[1] * es) % 16 == 0 and (chunk * es) % 16 == 0 and chunk * es > 4096)

    def close(self):
        """Unmap the peers' buffers (collective: no rank may still be writing into another's)."""
        import torch
        import torch.distributed as td

        if self.peers is None:
            return
        torch.cuda.synchronize(self.buffer.device)
        td.barrier(group=self.group)
        for base in self._opened:
            self._lib.nb200_ipc_close(ctypes.c_void_p(base))
        self._opened = []
        self.peers = None


def sharded_split_fold(name, x_shard, ncols_total: int, *, params=None, chunk: int = 16384, group=None,
                       partial_fn=None, merge_fn=None, widths=None, exchange=None, check: bool = False,
                       fused: bool | None = None):
    """Fold rows whose columns are sharded across the ranks of `group`, rank order = column order.

    Each rank passes its own [rows, width_r] block (the ranks' blocks concatenated along columns in
    rank order form the full rows). Returns out[rows] in x's dtype on every rank. Communication: one
    all-gather of the per-row chunk states (16 bytes per state). Shards of unequal width are padded
    with empty states, which the merge skips.

    `partial_fn(name, params, x_shard, col_begin, ncols_total, chunk) -> int32 [rows, nparts, 4]` and
    `merge_fn(name, params, states, out)` default to the CUDA kernels; tests on CPU ranks substitute
    their own to exercise the sharding and exchange logic. `widths` (every rank's shard width, in
    rank order) skips the width exchange -- and its host synchronisation -- when the caller knows
    the layout, as a steady-state loop does. With `exchange` (a PeerExchange whose slot width is the
    largest rank's chunk count) the states move through NVLink peer memory instead of an
    all-gather; the result is the same bit for bit -- in two launches (`PeerExchange.fold`: the fold
    stores into the peers' buffers itself) when the shard is contiguous and aligned and `fused` is
    set, else as a partial fold plus the exchange's push and merge kernels. `fused=None` picks by
    the group size as measured on B200 (bf16 [512, 262144], 16384-column chunks): the two-launch
    form at 2 ranks (43.6 vs 46.1 µs per call), the three-launch form at 8 (29.2 vs 41.0 µs), where
    every rank's fold storing into seven peers' buffers costs more than one push kernel. A merge whose bounded
    wait ran out writes its rows as NaN rather than leaving stale memory; `check=True` synchronises after
    the merge and raises if a wait ran out or a layout differed (marking the exchange unusable).
    """
    import torch
    import torch.distributed as td

    from neptune_opt_b200.skeletons import SKELETONS

    if SKELETONS[name].two_pass:
        raise NotImplementedError("two_pass needs extended carried state; split refused")
    partial_fn = partial_fn or _cuda_partial
    merge_fn = merge_fn or _cuda_merge
    world = td.get_world_size(group)
    rank = td.get_rank(group)
    rows, width = x_shard.shape
    if widths is None:
        mine = torch.tensor([width], dtype=torch.int64, device=x_shard.device)
        gathered_w = [torch.zeros_like(mine) for _ in range(world)]
        td.all_gather(gathered_w, mine, group=group)
        all_widths = [int(w.item()) for w in gathered_w]
    else:
        all_widths = [int(w) for w in widths]
        if len(all_widths) != world or all_widths[rank] != width:
            raise ValueError(f"widths {all_widths} do not describe rank {rank}'s shard of width {width}")
    if sum(all_widths) != ncols_total:
        raise ValueError(f"column shards sum to {sum(all_widths)}, expected {ncols_total}")
    col_begin = sum(all_widths[:rank])
    max_parts = max(-(-w // chunk) for w in all_widths)
    if exchange is not None:
        if exchange.nparts != max_parts or exchange.world != world:
            raise ValueError(f"the exchange holds {exchange.nparts} parts per rank for {exchange.world} ranks; "
                             f"this layout needs {max_parts} for {world}")
        out = torch.empty(rows, dtype=x_shard.dtype, device=x_shard.device)  # rows the merge cannot produce read NaN
        if fused is None:
            fused = world <= 2
        if fused and partial_fn is _cuda_partial and exchange.fold_eligible(x_shard, chunk):
            exchange.fold(name, params, x_shard, ncols_total, chunk, out)
        else:
            local = partial_fn(name, params, x_shard, col_begin, ncols_total, chunk)
            exchange.exchange_and_merge(name, params, local, out)
        if check:
            from neptune_opt_b200 import _lib

            bits = _lib.stream_fault()
            if bits & 0xC:
                exchange.faulted = True
                raise RuntimeError(f"peer exchange fault (bits {bits:#x}): "
                                   + ("a rank's states never arrived; " if bits & 4 else "")
                                   + ("a buffer's layout differs from the call's; " if bits & 8 else "")
                                   + "close the exchange on every rank and set up a new one")
        return out
    local = partial_fn(name, params, x_shard, col_begin, ncols_total, chunk)
    if local.shape[1] < max_parts:  # pad with empty (seen = 0) states
        pad = torch.zeros(rows, max_parts - local.shape[1], 4, dtype=local.dtype, device=local.device)
        pad[..., 0] = torch.tensor(float("-inf")).view(torch.int32) if local.dtype == torch.int32 else 0
        local = torch.cat([local, pad], dim=1)
    gathered = torch.empty((world * rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    td.all_gather_into_tensor(gathered, local.contiguous(), group=group)
    gathered = gathered.view((world,) + tuple(local.shape))
    # [world, rows, parts, 4] -> [rows, world * parts, 4]: ascending rank, then ascending chunk
    states = gathered.permute(1, 0, 2, 3).reshape(rows, world * max_parts, 4).contiguous()
    out = torch.empty(rows, dtype=x_shard.dtype, device=x_shard.device)
    return merge_fn(name, params, states, out)
