#!/usr/bin/env python
"""Throughput of neptune-opt's fused dependent-reduction regions on B200 (sm_100a kernels).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Headline workload: RMSNorm bf16 x[16384, 4096], gamma[4096], eps 1e-6;
one step = one fused RMSNorm pass over the batch. Every rank processes its own full batch (rows are
independent, no data-path collective): weak scaling, `value` = all ranks' algorithmic bytes / the
max-over-ranks step time. The other configs are measured after the headline and reported compactly
under `roofline.regions` (ms per step, aggregate GB/s or TFLOP/s, the per-GPU fraction of the
measured peak, ncu DRAM bytes per launch): softmax+logsumexp fp32, logsumexp fp32, L2-normalize
fp16, split-plan logsumexp bf16, ordered segment sum/mean fp16, and the fused tcgen05 attention bf16
[8,32,4096,128] non-causal and causal (burst and sustained, with torch SDPA on the same inputs as
library context). With N > 1 GPUs the strong-scaled partitions follow: RMSNorm rows, segment
blocks and attention heads of one fixed configuration, and the column-sharded split plan over NCCL
and over NVLink peer memory. Workload descriptions go to stderr (`bench detail`).

Algorithmic bytes count every tensor once (inputs read + outputs written). Between timed steps the
inputs rotate over buffer sets whose total exceeds the 126 MB L2, so no step reads data a previous
step left in L2. Times are CUDA events on the launching stream; the maximum over ranks is reported.

`--impl reference` times the reference's own CPU path for the headline: its unfused ATen RMSNorm
graph (restated op for op in oracle/aten_graph.py and bit-identical to the reference's outputs) on
torch's CPU kernels with all host threads, over the full batch per step. `cpu_baseline` reports the
same path, with the C restatement's (oracle/oracle.c) figure beside it.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "achieved HBM GB/s (% of 8 TB/s) & rows/s per fused region; attention TFLOP/s"
NOMINAL_HBM_GBS = 8000.0
L2_BYTES = 126 * 2**20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-regions", action="store_true", help="headline only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--region", default=None,
                    help="time one region only (rms_norm, softmax_lse, logsumexp, l2_normalize, "
                         "wide_logsumexp_split, wide_logsumexp_split_1024, segment_sum, segment_mean, attention, "
                         "attention_causal, "
                         "lse_1x262144, rms_1x65536, lse_256x16384) "
                         "and print its line; "
                         "used for ncu captures of a single kernel")
    ap.add_argument("--attention-batch", type=int, default=8,
                    help="batch of the attention regions (8 = the benchmark configuration; smaller "
                         "values only for profiler captures)")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(kernel_tag: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (line `traffic_bytes_per_launch[tag]: N`)."""
    for name in sorted(os.listdir(os.path.join(ROOT, "profiles"))) if os.path.isdir(os.path.join(ROOT, "profiles")) else []:
        if not name.endswith((".md", ".txt")):
            continue
        with open(os.path.join(ROOT, "profiles", name)) as f:
            for line in f:
                m = re.match(r"\s*traffic_bytes_per_launch\[(.+?)\]:\s*([0-9,]+)", line)
                if m and m.group(1) == kernel_tag:
                    return int(m.group(2).replace(",", ""))
    return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="nb200_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts)
        os.unlink(self.path)
        loaded = [r for r in rows if _num(r[4]) and _num(r[4]) > 0] or rows
        sm = [_num(r[1]) for r in loaded if _num(r[1])]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in loaded:
            for name, val in zip(names, r[6:10]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max((_num(r[2]) for r in rows if _num(r[2])), default=None),
                "power_w_max": max((_num(r[3]) for r in loaded if _num(r[3])), default=None),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded)}


def _num(s):
    try:
        return float(s)
    except (TypeError, ValueError):
        return None


# ---------------------------------------------------------------- distributed plumbing
class Dist:
    def __init__(self, n_gpus: int):
        import torch

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.n_gpus = n_gpus
        self.torch = torch
        self.pg = False
        if self.world > 1:
            import torch.distributed as td

            torch.cuda.set_device(self.local)
            td.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                  device_id=torch.device("cuda", self.local))
            self.pg = True
        elif torch.cuda.is_available():
            torch.cuda.set_device(0)

    def barrier(self):
        if self.pg:
            import torch.distributed as td

            td.barrier()

    def max(self, value: float) -> float:
        if not self.pg:
            return value
        import torch.distributed as td

        t = self.torch.tensor([value], dtype=self.torch.float64, device="cuda")
        td.all_reduce(t, op=td.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as td

            td.destroy_process_group()


# ---------------------------------------------------------------- workloads
def make_rms(torch, NB, seed):
    rows, ncols = 16384, 4096
    g = torch.Generator(device="cuda").manual_seed(seed)
    per = 2 * rows * ncols * 2
    nbuf = max(2, -(-3 * L2_BYTES // per) + 1)
    xs = [torch.randn(rows, ncols, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(nbuf)]
    outs = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    gamma = (1 + 0.1 * torch.randn(ncols, device="cuda", generator=g)).to(torch.bfloat16)

    def step(i):
        k = i % nbuf
        NB.template.launch_rms_norm(xs[k], gamma, outs[k], eps=1e-6)

    return {"name": "rms_norm", "step": step, "bytes": rows * ncols * 2 * 2 + ncols * 2, "rows": rows,
            "launches": 1, "buffers": nbuf, "io0": {"x": xs[0], "gamma": gamma, "y": outs[0]},
            "desc": f"rms_norm bf16 x[{rows},{ncols}] gamma[{ncols}] eps=1e-6 -> bf16 [{rows},{ncols}]"}


def make_softmax(torch, NB, seed):
    rows, ncols = 8192, 2048
    g = torch.Generator(device="cuda").manual_seed(seed)
    per = rows * ncols * 4 * 2
    nbuf = max(2, -(-3 * L2_BYTES // per) + 1)
    xs = []
    for _ in range(nbuf):
        x = torch.randn(rows, ncols, device="cuda", generator=g) * 2.0
        x[::64, 0] = 80.0
        xs.append(x)
    ys = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    lse = torch.empty(rows, device="cuda")
    lib = NB._lib.load()
    import ctypes

    def step(i):
        k = i % nbuf
        rc = lib.nb200_softmax(0, ctypes.c_void_p(xs[k].data_ptr()), 0, rows, ncols, ncols, 1,
                               ctypes.c_void_p(ys[k].data_ptr()), ctypes.c_void_p(lse.data_ptr()), None,
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        NB._lib.check(rc, "softmax")

    return {"name": "softmax_lse", "step": step, "bytes": rows * ncols * 4 * 2 + rows * 4, "rows": rows,
            "launches": 1, "buffers": nbuf, "io0": {"x": xs[0], "y": ys[0], "lse": lse},
            "desc": f"softmax + logsumexp fp32 x[{rows},{ncols}] N(0,2^2), every 64th row +80 -> y[{rows},{ncols}], lse[{rows}]"}


def make_lse(torch, NB, seed):
    rows, ncols = 8192, 2048
    g = torch.Generator(device="cuda").manual_seed(seed)
    per = rows * ncols * 4
    nbuf = max(2, -(-3 * L2_BYTES // per) + 1)
    xs = []
    for _ in range(nbuf):
        x = torch.randn(rows, ncols, device="cuda", generator=g) * 2.0
        x[::64, 0] = 80.0
        xs.append(x)
    out = torch.empty(rows, device="cuda")

    def step(i):
        k = i % nbuf
        NB.template.launch_reduction("logsumexp", "serial", xs[k], out, rows, ncols, None, None, {"tiny": 0.0})

    return {"name": "logsumexp", "step": step, "bytes": rows * ncols * 4 + rows * 4, "rows": rows, "launches": 1,
            "buffers": nbuf, "io0": {"x": xs[0], "out": out}, "desc": f"logsumexp fp32 x[{rows},{ncols}] -> [{rows}]"}


def make_l2(torch, NB, seed):
    rows, ncols = 65536, 768
    g = torch.Generator(device="cuda").manual_seed(seed)
    per = rows * ncols * 2 * 2
    nbuf = max(2, -(-3 * L2_BYTES // per) + 1)
    xs = [torch.randn(rows, ncols, device="cuda", dtype=torch.float16, generator=g) for _ in range(nbuf)]
    ys = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    norm = torch.empty(rows, device="cuda", dtype=torch.float16)
    lib = NB._lib.load()
    import ctypes

    def step(i):
        k = i % nbuf
        rc = lib.nb200_l2_normalize(ctypes.c_void_p(xs[k].data_ptr()), 2, rows, ncols, ncols, 1,
                                    ctypes.c_void_p(ys[k].data_ptr()), ctypes.c_void_p(norm.data_ptr()), None,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        NB._lib.check(rc, "l2")

    return {"name": "l2_normalize", "step": step, "bytes": rows * ncols * 2 * 2 + rows * 2, "rows": rows,
            "launches": 1, "buffers": nbuf, "io0": {"x": xs[0], "y": ys[0], "norm": norm}, "desc": f"L2-normalize fp16 x[{rows},{ncols}] -> y, norm"}


def make_wide_lse(torch, NB, seed, block=16384):
    """BASELINE config 3b: the split plan in 16384-column chunks; block=1024 is the reference's
    default split BLOCK (what its front end emits), on the same input."""
    rows, ncols = 512, 262144
    g = torch.Generator(device="cuda").manual_seed(seed)
    nbuf = 2
    xs = [(torch.randn(rows, ncols, device="cuda", generator=g) * 3.0).to(torch.bfloat16) for _ in range(nbuf)]
    out = torch.empty(rows, device="cuda", dtype=torch.bfloat16)

    def step(i):
        NB.template.launch_reduction("logsumexp", "split", xs[i % nbuf], out, rows, ncols, block, 8, {"tiny": 0.0})

    return {"name": "wide_logsumexp_split" + ("" if block == 16384 else f"_{block}"), "step": step,
            "bytes": rows * ncols * 2 + rows * 2, "rows": rows,
            "launches": 2, "buffers": nbuf, "io0": {"x": xs[0], "out": out},
            "desc": f"logsumexp bf16 x[{rows},{ncols}] N(0,3^2), split plan {block}-column chunks -> [{rows}]"}


def make_segments(torch, NB, seed, reduce="sum"):
    nseg, channels = 200000, 128
    gen = torch.Generator().manual_seed(0)
    lengths = torch.poisson(torch.full((nseg,), 20.0), generator=gen).clamp(1, 200).to(torch.int64)
    offsets = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)]).cuda()
    T = int(lengths.sum())
    g = torch.Generator(device="cuda").manual_seed(seed)
    data = torch.randn(T, channels, device="cuda", dtype=torch.float16, generator=g)
    from neptune_opt_b200.torch_op import _launch_segment

    params = {"initial": None, "offsets": True, "unsafe": False}
    last = {}

    def step(i):
        last["out"] = _launch_segment("segment_" + reduce, data, offsets, params, "serial")

    return {"name": f"segment_{reduce}", "step": step,
            "bytes": T * channels * 2 + (nseg + 1) * 8 + nseg * channels * 2, "rows": nseg, "launches": 1,
            "buffers": 1, "T": T, "io0": {"data": data, "offsets": offsets, "lengths": lengths, "last": last},
            "desc": f"ordered segment_{reduce} fp16 data[{T},{channels}], {nseg} segments Poisson(20) in [1,200], int64 offsets"}


def make_attention(torch, NB, seed, causal=False, batch=8):
    b, h, s, d = batch, 32, 4096, 128
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(b, h, s, d, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(3))
    o = torch.empty_like(q)
    lse = torch.empty(b, h, s, device="cuda", dtype=torch.float32)
    from neptune_opt_b200.attention import launch_attention

    def step(_i):
        launch_attention(q, k, v, o, lse, causal=causal, scale=1.0 / d ** 0.5)

    pairs = s * s if not causal else s * (s + 1) // 2  # (query, key) pairs attended per head
    name = "attention_causal" if causal else "attention"
    return {"name": name, "step": step, "flops": 4 * b * h * d * pairs, "rows": b * h * s, "launches": 1,
            "bytes": 4 * b * h * s * d * 2 + b * h * s * 4, "buffers": 1,
            "desc": f"attention bf16 q,k,v[{b},{h},{s},{d}] N(0,1), scale 1/sqrt({d}), "
                    f"{'causal' if causal else 'non-causal'} -> o bf16, lse fp32 (inputs {3 * b * h * s * d * 2 >> 20} MiB > L2)"}


def make_small(torch, NB, seed, kind):
    """The reference's published small shapes (README: logsumexp fp32 (1, 262144), RMSNorm fp32
    (1, 65536), logsumexp fp32 256 x 16384) through the library's default launch, and for the two
    single rows the launches they replace: the split plan's two launches (16K-column chunks, then
    the merge) and one CTA of 512 threads per row. Inputs rotate over more than 126 MB."""
    import ctypes

    lib = NB._lib.load()
    rows, ncols = {"lse_1x262144": (1, 262144), "rms_1x65536": (1, 65536), "lse_256x16384": (256, 16384)}[kind]
    g = torch.Generator(device="cuda").manual_seed(seed)
    per = rows * ncols * 4
    nbuf = max(2, -(-L2_BYTES // per) + 1)
    xs = [torch.randn(rows, ncols, device="cuda", generator=g) * 2.0 for _ in range(nbuf)]
    out = torch.empty(rows, ncols, device="cuda") if kind.startswith("rms") else torch.empty(rows, device="cuda")
    gamma = 1 + 0.1 * torch.randn(ncols, device="cuda", generator=g)
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    cta = NB._lib.launch_struct(NB._lib.VARIANT_CTA_ROW, 512, 0, 0)

    def step_for(how):
        def step(i):
            x = xs[i % nbuf]
            if kind.startswith("rms"):
                NB.template.launch_rms_norm(x, gamma, out, eps=1e-6, launch=cta if how == "cta_row" else None)
            elif how == "split":
                NB.template.launch_reduction("logsumexp", "split", x, out, rows, ncols, 16384, 8, {"tiny": 0.0})
            elif how == "cta_row":
                p = NB._lib.params_struct({"tiny": 0.0})
                NB._lib.check(lib.nb200_fold(0, ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), 0, rows, ncols, ncols,
                                             1, ctypes.c_void_p(out.data_ptr()), ctypes.byref(cta), stream()), "fold")
            else:
                NB.template.launch_reduction("logsumexp", "serial", x, out, rows, ncols, None, None, {"tiny": 0.0})
        return step

    nbytes = rows * ncols * 4 * (2 if kind.startswith("rms") else 1) + (ncols * 4 if kind.startswith("rms") else rows * 4)
    return {"name": kind, "step": step_for("default"), "bytes": nbytes, "rows": rows, "launches": 1, "buffers": nbuf,
            "alternatives": {} if rows > 1 else {"split_ms": step_for("split"), "cta_row_ms": step_for("cta_row")},
            "desc": f"{'rms_norm' if kind.startswith('rms') else 'logsumexp'} fp32 [{rows},{ncols}] (reference README shape)"}


def make_sharded_split(torch, NB, seed, dist, peer=False, fused=True):
    """BASELINE config 3b across GPUs: the columns of bf16 [512, 262144] split into one shard per
    rank; each rank folds its shard into 16K-column chunk states, which move to every rank -- one
    NCCL all-gather, or (peer=True) epoch-tagged stores into every rank's exchange buffer over
    NVLink -- and every rank merges them in ascending (rank, chunk) order. Total work is fixed
    (strong scaling)."""
    from neptune_opt_b200.parallel import PeerExchange, sharded_split_fold

    rows, ncols, block = 512, 262144, 16384
    n = dist.world
    width = ncols // n
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = [(torch.randn(rows, width, device="cuda", generator=g) * 3.0).to(torch.bfloat16) for _ in range(2)]
    ex = None
    if peer:
        try:  # set-up decides on every rank together (it raises on all ranks or on none)
            ex = PeerExchange(rows, -(-width // block))
        except Exception as exc:  # noqa: BLE001
            if dist.rank == 0:
                print(f"peer exchange unavailable, region skipped: {exc}", file=sys.stderr, flush=True)
            return None

    def step(i):
        sharded_split_fold("logsumexp", xs[i % 2], ncols, params={"tiny": 0.0}, chunk=block, widths=[width] * n,
                           exchange=ex, fused=fused)

    how = (("two launches: fold storing epoch-tagged states into every rank's exchange buffer over NVLink; "
            "merge reads each state until it carries the call's epoch" if fused else "partial fold, push kernel "
            "(epoch-tagged stores into every rank's buffer), merge kernel (reads each state until tagged)")
           if peer else "states all-gathered over NCCL")
    name = "wide_logsumexp_split_sharded" + (("_peer" if fused else "_peer_3launch") if peer else "")
    return {"name": name, "step": step,
            "bytes": rows * ncols * 2 + rows * 2, "rows": rows, "launches": (2 if fused else 3) if peer else 2,
            "buffers": 2,
            "exchange": ex,
            "desc": f"logsumexp bf16 x[{rows},{ncols}] N(0,3^2), columns sharded over {n} GPUs ({width} each), "
                    f"{block}-column chunk states {how}, merged in rank order"}


def make_rms_rows_sharded(torch, NB, seed, dist):
    """BASELINE config 2 strong-scaled: the [16384, 4096] bf16 batch's rows split into one
    contiguous block per rank (parallel.shard_rows); no data-path collective."""
    from neptune_opt_b200.parallel import shard_rows

    rows, ncols = 16384, 4096
    b, e = shard_rows(rows, dist.world, dist.rank)
    local = e - b
    g = torch.Generator(device="cuda").manual_seed(seed)
    nbuf = max(2, -(-3 * L2_BYTES // (2 * local * ncols * 2)) + 1)
    xs = [torch.randn(local, ncols, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(nbuf)]
    outs = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    gamma = (1 + 0.1 * torch.randn(ncols, device="cuda", generator=g)).to(torch.bfloat16)

    def step(i):
        NB.template.launch_rms_norm(xs[i % nbuf], gamma, outs[i % nbuf], eps=1e-6)

    return {"name": "rms_norm_rows_sharded", "step": step, "bytes": rows * ncols * 4 + ncols * 2, "rows": rows,
            "launches": 1, "buffers": nbuf,
            "desc": f"rms_norm bf16 [16384,4096], rows sharded over {dist.world} GPU(s) ({local} here)"}


def make_segments_sharded(torch, NB, seed, dist, reduce="sum"):
    """BASELINE config 4 strong-scaled: whole segments in contiguous blocks whose token counts
    balance (parallel.shard_segments); each rank pools its block, bit-exact, no collective."""
    from neptune_opt_b200.parallel import local_offsets, shard_segments
    from neptune_opt_b200.torch_op import _launch_segment

    nseg, channels = 200000, 128
    gen = torch.Generator().manual_seed(0)
    lengths = torch.poisson(torch.full((nseg,), 20.0), generator=gen).clamp(1, 200).to(torch.int64)
    offsets = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)])
    T = int(offsets[-1])
    shard = shard_segments(offsets, dist.world, dist.rank)
    local_off = local_offsets(offsets, shard).cuda()
    g = torch.Generator(device="cuda").manual_seed(seed)
    data = torch.randn(shard.row_end - shard.row_begin, channels, device="cuda", dtype=torch.float16, generator=g)
    params = {"initial": None, "offsets": True, "unsafe": False}

    def step(i):
        _launch_segment("segment_" + reduce, data, local_off, params, "serial")

    return {"name": f"segment_{reduce}_sharded", "step": step,
            "bytes": T * channels * 2 + (nseg + 1) * 8 + nseg * channels * 2, "rows": nseg, "launches": 1,
            "buffers": 1,
            "desc": f"segment_{reduce} fp16 [{T},128], 200000 segments in token-balanced blocks over "
                    f"{dist.world} GPU(s) ({shard.seg_end - shard.seg_begin} here)"}


def make_attention_sharded(torch, NB, seed, dist, causal=False):
    """BASELINE config 5 strong-scaled: the 8 x 32 (batch, head) pairs split into contiguous blocks
    (parallel.shard_heads), each rank running its block as one [1, pairs, 4096, 128] launch."""
    from neptune_opt_b200.attention import launch_attention
    from neptune_opt_b200.parallel import shard_heads

    b, h, s, d = 8, 32, 4096, 128
    lo, hi = shard_heads(b, h, dist.world, dist.rank)
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(1, hi - lo, s, d, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(3))
    o = torch.empty_like(q)
    lse = torch.empty(1, hi - lo, s, device="cuda", dtype=torch.float32)

    def step(_i):
        launch_attention(q, k, v, o, lse, causal=causal, scale=1.0 / d ** 0.5)

    pairs = s * s if not causal else s * (s + 1) // 2
    return {"name": "attention" + ("_causal" if causal else "") + "_heads_sharded", "step": step,
            "flops": 4 * b * h * d * pairs, "rows": b * h * s, "launches": 1, "buffers": 1,
            "desc": f"attention bf16 [8,32,4096,128]{' causal' if causal else ''}, (batch, head) pairs sharded "
                    f"over {dist.world} GPU(s) ({hi - lo} here)"}


def sdpa_tflops(torch, causal, flops):
    """torch's scaled_dot_product_attention (library kernels) on the same [8,32,4096,128] bf16
    inputs, 10 launches between CUDA events: context for the attention regions."""
    import torch.nn.functional as F

    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v = (torch.randn(8, 32, 4096, 128, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(3))
    for _ in range(3):
        F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(10):
        F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / 10
    del q, k, v
    return round(flops / (ms * 1e-3) / 1e12, 1)


def gpu_id(torch) -> str:
    """nvidia-smi id of the current device (PCI bus id when torch exposes it)."""
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    bus = getattr(props, "pci_bus_id", None)
    if bus is not None:
        return f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:{getattr(props, 'pci_device_id', 0):02x}.0"
    return str(torch.cuda.current_device())


def time_steps(torch, dist, step, steps, warmup, graph=True):
    """(max-over-ranks ms per step, kernel launches in the timed region).

    graph=True: the K steps are captured once into a CUDA graph (each step's real launches, inputs
    rotating as in eager execution) and the graph is replayed once between CUDA events, so the time
    is the device's, free of Python launch overhead. graph=False times K eager calls."""
    import neptune_opt_b200 as NB

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    g = None
    n0 = NB.launch_count()
    if graph:
        g = torch.cuda.CUDAGraph()
        capture = torch.cuda.Stream()
        capture.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=capture):
            for i in range(steps):
                step(warmup + i)
        launches = NB.launch_count() - n0
        g.replay()  # untimed first replay (graph upload)
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    if graph:
        g.replay()
    else:
        for i in range(steps):
            step(warmup + i)
    end.record()
    torch.cuda.synchronize()
    if not graph:
        launches = NB.launch_count() - n0
    dist.barrier()
    ms = start.elapsed_time(end) / steps
    del g
    return dist.max(ms), launches


def tensor_roofline(flops_per_launch, ms, peaks, traffic):
    achieved = flops_per_launch / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4),
            "peak_source": peaks["source"] + " (burst cuBLAS bf16 GEMM)", "traffic": traffic}


def time_collective_steps(torch, dist, step, steps, warmup):
    """Max-over-ranks ms per step of a step that holds NCCL collectives.

    Every rank runs the warm-up eagerly, then tries to capture the K steps into one CUDA graph
    (capture records the collectives without running them). The ranks agree on the outcome with an
    eager all-reduce before anything is replayed, so all of them either replay their graphs or all
    time eager steps: the collectives stay matched on every path."""
    import torch.distributed as td

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    g, ok = torch.cuda.CUDAGraph(), 1
    try:
        capture = torch.cuda.Stream()
        capture.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=capture):
            for i in range(steps):
                step(warmup + i)
    except Exception:  # noqa: BLE001 -- decided jointly below
        ok = 0
    torch.cuda.synchronize()
    flag = torch.tensor([ok], dtype=torch.int32, device="cuda")
    td.all_reduce(flag, op=td.ReduceOp.MIN)
    graph = bool(flag.item())
    if graph:
        g.replay()  # untimed first replay
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    if graph:
        g.replay()
    else:
        for i in range(steps):
            step(warmup + i)
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    del g
    how = ("CUDA graph (the step's kernels and collectives captured together)" if graph
           else "eager (graph capture was not possible on every rank)") + ", max over ranks"
    return dist.max(start.elapsed_time(end) / steps), how


def roofline(bytes_per_launch, ms, peaks, traffic):
    achieved = bytes_per_launch / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"] + " (burst copy)",
            "frac_of_nominal": round(achieved / NOMINAL_HBM_GBS, 4),  # BASELINE's "% of 8 TB/s"
            "traffic": traffic}


# ---------------------------------------------------------------- CPU legs (reference path on the host)
def _host_rms_inputs(rows, ncols, seed=0):
    """Seeded host copies of the headline inputs: x bf16 ~ N(0,1), gamma bf16 ~ N(1, 0.1)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, ncols, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(ncols, generator=g)).to(torch.bfloat16)
    return x, gamma


def _host_threads():
    """Use every host core for the CPU legs; returns the thread count torch will use."""
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    return torch.get_num_threads()


def time_aten_rms(steps: int, warmup: int, budget_s: float):
    """The reference's unfused ATen RMSNorm graph (oracle/aten_graph.py, bit-identical to the
    reference's outputs) on the host: (seconds per step, rows per step, threads). Each step is the
    full [16384, 4096] batch unless `steps` full passes would exceed `budget_s`, in which case each
    step is a leading row block sized to fit (declared by the caller)."""
    import time as _t

    from oracle import aten_graph

    threads = _host_threads()
    rows, ncols = 16384, 4096
    x, gamma = _host_rms_inputs(rows, ncols)
    t0 = _t.perf_counter()
    aten_graph.rms_norm(x, gamma, 1e-6)
    first = _t.perf_counter() - t0
    sample = rows
    if first * (steps + warmup) > budget_s:
        sample = max(256, int(rows * budget_s / (first * (steps + warmup))) // 256 * 256)
    xs = x[:sample]
    for _ in range(max(0, warmup - 1)):
        aten_graph.rms_norm(xs, gamma, 1e-6)
    t0 = _t.perf_counter()
    for _ in range(steps):
        aten_graph.rms_norm(xs, gamma, 1e-6)
    return (_t.perf_counter() - t0) / steps, sample, threads


def time_c_port_rms(seconds: float):
    """The C restatement (oracle/oracle.c, OpenMP over all host threads) over the full headline
    batch, repeated for about `seconds`: (GB/s at bf16 bytes, threads, passes)."""
    import numpy as np

    import oracle

    rows, ncols = 16384, 4096
    x, gamma = _host_rms_inputs(rows, ncols)
    xf, gf = x.float().numpy(), gamma.float().numpy()
    oracle.rms_norm(xf[:64], gf, 1e-6, "bfloat16")  # load + warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.rms_norm(xf, gf, 1e-6, "bfloat16")
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    del np
    return reps * (rows * ncols * 4 + ncols * 2) / dt / 1e9, oracle.num_threads(), reps


RMS_BYTES_PER_ROW = 4096 * 2 * 2  # read x + write y, bf16
ATEN_PATH = ("the reference's unfused ATen RMSNorm graph on the host (tests/test_recognize.py:595-597 form, "
             "oracle/aten_graph.py, bit-identical to the reference's outputs), torch CPU kernels")


def cpu_baseline_rms(seconds: float):
    """cpu_baseline of the headline: the reference's ATen graph on host cores, with the C port's
    figure beside it."""
    steps = 8
    dt, sample, threads = time_aten_rms(steps, 1, seconds)
    value = sample * RMS_BYTES_PER_ROW / dt / 1e9
    cport, cthreads, reps = time_c_port_rms(min(5.0, seconds / 2))
    return {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{steps} passes of {sample} of 16384 rows, the reference's ATen RMSNorm graph on host "
                      f"({dt * 1e3:.0f} ms/pass)",
            "c_port_GBps": round(cport, 3),
            "detail": {"path": ATEN_PATH,
                       "c_port": f"oracle/oracle.c restatement, {cthreads} OpenMP threads, {reps} full passes"}}


def run_reference(args):
    """`--impl reference`: the reference's CPU path for the headline on rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    dt, sample, threads = time_aten_rms(args.steps, args.warmup, 150.0)
    value = sample * RMS_BYTES_PER_ROW / dt / 1e9
    full = sample == 16384
    desc = ("full batch" if full else f"leading {sample} of the 16384 rows (the full batch per step would "
            f"exceed the time budget)")
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) x, N(1,0.1) gamma)",
            "config": {"workload": "rms_norm bf16 x[16384,4096] gamma[4096] eps=1e-6 -> bf16 [16384,4096]",
                       "rows_per_step": sample, "ncols": 4096, "path": ATEN_PATH},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{desc} per step, {args.steps} timed steps after {args.warmup} warm-up"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "rows_per_s": round(sample / dt, 1)}
    print(json.dumps(line), flush=True)
    return 0


REGION_MAKERS = {
    "rms_norm": make_rms, "softmax_lse": make_softmax, "logsumexp": make_lse, "l2_normalize": make_l2,
    "wide_logsumexp_split": make_wide_lse,
    "wide_logsumexp_split_1024": lambda t, nb, s: make_wide_lse(t, nb, s, block=1024),
    "segment_sum": lambda t, nb, s: make_segments(t, nb, s, "sum"),
    "segment_mean": lambda t, nb, s: make_segments(t, nb, s, "mean"),
    "attention": make_attention,
    "attention_causal": lambda t, nb, s, **kw: make_attention(t, nb, s, causal=True, **kw),
    "lse_1x262144": lambda t, nb, s: make_small(t, nb, s, "lse_1x262144"),
    "rms_1x65536": lambda t, nb, s: make_small(t, nb, s, "rms_1x65536"),
    "lse_256x16384": lambda t, nb, s: make_small(t, nb, s, "lse_256x16384"),
}
REGION_OPTIONS = {"attention": ("attention_batch", "batch"), "attention_causal": ("attention_batch", "batch")}


def run_region(args, torch, NB, dist, peaks):
    kw = {}
    if args.region in REGION_OPTIONS:
        arg, key = REGION_OPTIONS[args.region]
        kw[key] = getattr(args, arg)
    r = REGION_MAKERS[args.region](torch, NB, 3000 + dist.rank, **kw)
    ms, launches = time_steps(torch, dist, r["step"], args.steps, max(3, args.warmup), graph=False)
    if dist.rank == 0:
        roof = (tensor_roofline(r["flops"], ms, peaks, None) if "flops" in r
                else roofline(r["bytes"] / r["launches"], ms / r["launches"], peaks, None))
        print(json.dumps({"region": r["name"], "workload": r["desc"], "ms_per_step": round(ms, 5),
                          "GB_per_s": round(dist.world * r["bytes"] / (ms * 1e-3) / 1e9, 1),
                          "roofline": roof, "gpu_launches": launches}), flush=True)
    dist.close()
    return 0


# ---------------------------------------------------------------- main
def hbm_region(r, ms, n, peaks, strong=False):
    """Compact record of an HBM-bound region: ms per step (max over ranks), aggregate GB/s, the
    per-GPU fraction of the measured copy peak, and ncu DRAM bytes per launch (profiles/)."""
    per_gpu = r["bytes"] / (n if strong else 1)
    rec = {"ms": round(ms, 5), "GBps": round((1 if strong else n) * r["bytes"] / (ms * 1e-3) / 1e9, 1),
           "frac": round(per_gpu / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
           "traffic": profile_traffic(r["name"]) if n == 1 else None}
    if strong:
        rec["strong"] = True
    return rec


def tensor_region(r, ms, n, peaks, strong=False, sustained_ms=None, sdpa=None):
    per_gpu = r["flops"] / (n if strong else 1)
    rec = {"ms": round(ms, 5), "TFLOPs": round((1 if strong else n) * r["flops"] / (ms * 1e-3) / 1e12, 1),
           "frac": round(per_gpu / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
           "traffic": profile_traffic(r["name"]) if n == 1 else None}
    if sustained_ms is not None:
        sus = per_gpu / (sustained_ms * 1e-3) / 1e12
        rec["sus_TFLOPs"] = round(sus * (1 if strong else n), 1)
        rec["sus_frac"] = round(sus / peaks["bf16_tflops_sustained"], 4)
    if sdpa is not None:
        rec["sdpa_TFLOPs"] = sdpa
    if strong:
        rec["strong"] = True
    return rec


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    import torch

    import neptune_opt_b200 as NB

    NB.load()
    dist = Dist(args.gpus)
    if args.region:
        return run_region(args, torch, NB, dist, load_peaks())
    peaks = load_peaks()
    n = dist.world
    sampler = ClockSampler(gpu_id(torch)).start() if dist.rank == 0 else None
    detail = {}

    # ---- headline: RMSNorm, every rank its own [16384, 4096] batch (weak scaling)
    w = make_rms(torch, NB, seed=1000 + dist.rank)
    ms, launches = time_steps(torch, dist, w["step"], args.steps, max(3, args.warmup))
    eager_ms, _ = time_steps(torch, dist, w["step"], args.steps, max(3, args.warmup), graph=False)
    value = n * w["bytes"] / (ms * 1e-3) / 1e9
    head_roof = roofline(w["bytes"] / w["launches"], ms / w["launches"], peaks, profile_traffic("rms_norm"))
    detail["rms_norm"] = {"workload": w["desc"], "eager_ms_per_step": round(eager_ms, 5)}
    del w
    torch.cuda.empty_cache()

    # ---- e2e through the public API with host buffers
    rows, ncols = 16384, 4096
    xh = torch.randn(rows, ncols, dtype=torch.bfloat16).pin_memory()
    gh = (1 + 0.1 * torch.randn(ncols)).to(torch.bfloat16).pin_memory()
    oh = torch.empty(rows, ncols, dtype=torch.bfloat16).pin_memory()

    def e2e_step(_i):
        # Rows stream through the GPU in 16 MiB chunks; the copies in and out of the device
        # overlap each other and the kernel (nb200_rms_norm_host).
        NB.run_rms_norm_host(xh, gh, eps=1e-6, out=oh)

    e2e_steps = max(3, min(args.steps, 30))
    e2e_ms, _ = time_steps(torch, dist, e2e_step, e2e_steps, 3, graph=False)
    e2e = {"value": round(n * (rows * ncols * 4 + ncols * 2) / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": rows * ncols * 2 + ncols * 2, "d2h_bytes_per_step": rows * ncols * 2,
           "ms_per_step": round(e2e_ms, 4), "steps": e2e_steps,
           "path": "pinned host -> run_rms_norm_host -> pinned host"}
    detail["e2e"] = ("pinned host x,gamma -> run_rms_norm_host (nb200_rms_norm_host, 16 MiB chunks, copies "
                     "overlapping the kernel) -> pinned host y")
    del xh, gh, oh

    # ---- the other configurations
    regions = {}
    if not args.no_regions:
        makers = [make_softmax, make_lse, make_l2, make_wide_lse,
                  lambda t, nb, s: make_wide_lse(t, nb, s, block=1024),
                  lambda t, nb, s: make_segments(t, nb, s, "sum"), lambda t, nb, s: make_segments(t, nb, s, "mean")]
        for maker in makers:
            r = maker(torch, NB, 2000 + dist.rank)
            rms_, _ = time_steps(torch, dist, r["step"], args.steps, max(3, args.warmup))
            regions[r["name"]] = hbm_region(r, rms_, n, peaks)
            detail[r["name"]] = {"workload": r["desc"], "launches_per_step": r["launches"],
                                 "l2_rotation_buffers": r["buffers"],
                                 "rows_per_s": round(n * r["rows"] / (rms_ * 1e-3), 1)}
            del r
            torch.cuda.empty_cache()
        for kind in ("lse_1x262144", "rms_1x65536", "lse_256x16384"):
            r = make_small(torch, NB, 2300 + dist.rank, kind)
            sms_, _ = time_steps(torch, dist, r["step"], max(args.steps, 50), max(3, args.warmup))
            rec = hbm_region(r, sms_, n, peaks)
            for key, alt in r["alternatives"].items():
                if kind.startswith("rms") and key == "split_ms":
                    continue  # RMSNorm's split plan is the same one-launch kernel
                ams_, _ = time_steps(torch, dist, alt, max(args.steps, 50), max(3, args.warmup))
                rec[key] = round(ams_, 5)
            regions[r["name"]] = rec
            detail[r["name"]] = {"workload": r["desc"], "l2_rotation_buffers": r["buffers"]}
            del r
            torch.cuda.empty_cache()
        for causal in (False, True):
            # Burst: 10 launches (~20 ms), the regime of the burst GEMM peak. Sustained: 100
            # launches back to back (~0.2 s under the power cap), against the sustained peak.
            r = make_attention(torch, NB, 2500 + dist.rank, causal=causal)
            ams, _ = time_steps(torch, dist, r["step"], 10, max(3, args.warmup))
            sms, _ = time_steps(torch, dist, r["step"], 100, 3)
            sdpa = sdpa_tflops(torch, causal, r["flops"]) if dist.rank == 0 else None
            regions[r["name"]] = tensor_region(r, ams, n, peaks, sustained_ms=sms, sdpa=sdpa)
            detail[r["name"]] = {"workload": r["desc"]}
            del r
            torch.cuda.empty_cache()
        if n > 1:
            # strong scaling: one fixed BASELINE configuration partitioned over the ranks
            for maker, kind in ((make_rms_rows_sharded, "hbm"),
                                (lambda t, nb, s, d: make_segments_sharded(t, nb, s, d, "sum"), "hbm"),
                                (lambda t, nb, s, d: make_attention_sharded(t, nb, s, d, False), "tensor"),
                                (lambda t, nb, s, d: make_attention_sharded(t, nb, s, d, True), "tensor")):
                r = maker(torch, NB, 2700 + dist.rank, dist)
                steps = args.steps if kind == "hbm" else 10
                sms_, _ = time_steps(torch, dist, r["step"], steps, max(3, args.warmup))
                regions[r["name"]] = (hbm_region(r, sms_, n, peaks, strong=True) if kind == "hbm"
                                      else tensor_region(r, sms_, n, peaks, strong=True))
                detail[r["name"]] = {"workload": r["desc"]}
                del r
                torch.cuda.empty_cache()
            for peer, fused in ((False, True), (True, True), (True, False)):
                r = make_sharded_split(torch, NB, 2600, dist, peer=peer, fused=fused)
                if r is None:
                    continue
                steps = min(args.steps, 50)
                sms_, how = time_collective_steps(torch, dist, r["step"], steps, max(3, args.warmup))
                rec = hbm_region(r, sms_, n, peaks, strong=True)
                # a wait that ran out on any rank (fault bit) voids the region's timing on every rank
                fault = torch.tensor([NB._lib.stream_fault()], dtype=torch.int64, device="cuda")
                torch.distributed.all_reduce(fault, op=torch.distributed.ReduceOp.MAX)
                if int(fault.item()):
                    rec = {"fault": f"bounded wait ran out (bits {int(fault.item()):#x})"}
                regions[r["name"]] = rec
                detail[r["name"]] = {"workload": r["desc"], "timing": how}
                if r["exchange"] is not None:
                    r["exchange"].close()
                del r
                torch.cuda.empty_cache()
    clocks = sampler.stop() if sampler else None

    cpu = None
    if dist.rank == 0 and n == 1 and not args.no_cpu:
        try:
            cpu = cpu_baseline_rms(20.0)
        except Exception as exc:  # noqa: BLE001 -- the baseline is reported, never the measured value
            cpu = {"value": None, "unit": "GB/s", "cores": None, "kind": "port", "sample": f"failed: {exc}"}

    if dist.rank == 0:
        head_roof["regions"] = regions
        if cpu is not None and "detail" in cpu:
            detail["cpu_baseline"] = cpu.pop("detail")
        # roofline (with every region's record) goes last: a reader that keeps only the end of a long
        # line still has all of the measurements
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": n, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) x, N(1,0.1) gamma on device)",
            "config": {"workload": "rms_norm bf16 x[16384,4096] gamma[4096] eps=1e-6, per GPU",
                       "timing": "CUDA graph of K steps, CUDA events, max over ranks",
                       "l2": "inputs rotate over buffers > 3x L2"},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks, "roofline": head_roof,
        }
        print("bench detail " + json.dumps(detail), file=sys.stderr, flush=True)
        print(json.dumps(line), flush=True)
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
