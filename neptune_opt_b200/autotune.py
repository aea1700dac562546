"""Launch-configuration policy for the CUDA folds on B200.

The reference picks Triton meta-parameters `(BLOCK, num_warps)` per shape bucket from a per-GPU
measured table (neptune_codegen/autotune.py:222-250, table launch_table.py:23-49). This module keeps
that policy and its vocabulary -- a `(block, num_warps)` pair, `(rows class, pow2 width bucket)`
keys, a machine-keyed table holding only measured deviations from the default, a noise margin a
candidate must clear -- but the pair now selects a CUDA launch:

* ``num_warps == 0``: the library's own policy -- contiguous, 16-byte aligned rows of 1-8 KB are
  loaded whole into one warp's registers (several rows per CTA), rows of 8-32 KB are staged through
  shared memory with bulk copies (each warp owns a ring of stages), others use the register-tiled
  kernels below;
* ``num_warps == 1``: one warp folds one row (persistent CTAs of 8 warps, row chunks resident in
  registers, no shared memory or barriers);
* ``2 <= num_warps <= 16``: one CTA of ``32 * num_warps`` threads folds one row (cross-warp
  reduction through shared memory);
* ``num_warps == 32``: one thread-block cluster folds one row (up to 16 CTAs of 8 warps, their
  states merged through distributed shared memory in one launch; contiguous aligned rows);
* ``block`` is the split plan's chunk width in columns (one CTA per chunk). The serial kernels size
  their register tile from the row width themselves, so for the serial plan ``block`` only takes
  part in the operator's identity.

The default is the library's policy, `(SPLIT_BLOCK, 0)`.
"""
from __future__ import annotations

import dataclasses
import hashlib
import math

from neptune_opt_b200._lib import VARIANT_CLUSTER, VARIANT_CTA_ROW, VARIANT_WARP_ROW, launch_struct

# Every configuration the search may choose from.
CANDIDATES: tuple = (
    (16384, 0),
    (4096, 1), (16384, 1),
    (4096, 4), (16384, 4),
    (4096, 8), (16384, 8),
    (16384, 16),
    (16384, 32),
)

# The split plan's chunk width when nothing else is known: 16K columns per CTA (32 KB of bf16).
SPLIT_BLOCK = 16384
WARP_ROW_BYTES = 16384

MIN_BUCKET = 256
MAX_BUCKET = 1 << 22
THIN_ROWS = 8
NOISE = 0.05
MACHINE = "b200"


def machine_key(device_name: str | None = None) -> str:
    """Normalised GPU name: 'NVIDIA B200' -> 'b200'."""
    name = device_name
    if name is None:
        try:  # pragma: no cover - needs a GPU
            import torch

            if not torch.cuda.is_available():
                return ""
            name = torch.cuda.get_device_name(torch.cuda.current_device())
        except Exception:  # noqa: BLE001
            return ""
    words = []
    for word in str(name).lower().replace("+", " ").split():
        if word in ("nvidia", "geforce", "tesla", "graphics", "corporation"):
            continue
        words.append("".join(ch if ch.isalnum() else "-" for ch in word).strip("-"))
    return "-".join(w for w in words if w)


def ncols_bucket(ncols) -> int:
    if not isinstance(ncols, int):
        raise ValueError("a measured width bucket requires a static integer width")
    n = max(1, ncols)
    return max(MIN_BUCKET, min(MAX_BUCKET, 1 << (n - 1).bit_length()))


def rows_class(rows) -> str:
    if not isinstance(rows, int):
        return "many"
    if rows <= 1:
        return "single"
    return "few" if rows <= THIN_ROWS else "many"


def shape_key(rows, ncols) -> tuple:
    return rows_class(rows), ncols_bucket(ncols)


def _elem_bytes(dtype) -> int:
    text = str(dtype)
    return 4 if text.endswith("float32") or text == "float32" else 2


def default_config(ncols=None, dtype=None) -> tuple:
    """The library's launch policy (bulk-copy staging when eligible)."""
    return (SPLIT_BLOCK, 0)


DEFAULT = default_config()


def _module_tables() -> dict:
    try:
        from neptune_opt_b200 import launch_table
    except Exception:  # noqa: BLE001
        return {}
    out = {}
    for machine, entry in getattr(launch_table, "TABLES", {}).items():
        body = entry.get("table") or {}
        out[machine] = {**{k: v for k, v in entry.items() if k != "table"}, "table": _valid(body)}
    return out


def _valid(body) -> dict:
    return {tuple(k): tuple(v) for k, v in (body or {}).items() if tuple(v) in CANDIDATES}


def tables() -> dict:
    return _module_tables()


def table(machine: str | None = None) -> dict:
    """The measured deviations for one machine; never another machine's numbers."""
    all_tables = tables()
    if machine is None:
        machine = machine_key()
    return dict(all_tables.get(machine, {}).get("table", {}))


_NAMES: dict = {}


def _device_name(device: str):
    """The GPU name of a CUDA device string, cached (asked once per device)."""
    if device not in _NAMES:
        try:
            import torch

            _NAMES[device] = torch.cuda.get_device_name(torch.device(device))
        except Exception:  # noqa: BLE001
            _NAMES[device] = None
    return _NAMES[device]


def best_config(rows, ncols, dtype=None, device=None, device_name=None, verbose: bool = False) -> tuple:
    """`(block, num_warps)` for a shape on this machine: measured entry, else the default."""
    if not isinstance(rows, int) or not isinstance(ncols, int):
        return default_config(ncols if isinstance(ncols, int) else None, dtype)
    default = default_config(ncols, dtype)
    if device is not None and str(device).split(":", 1)[0] != "cuda":
        return default
    if device_name is None and device is not None:
        device_name = _device_name(str(device))
    machine = machine_key(device_name) if device_name else ""
    cfg = table(machine).get(shape_key(rows, ncols), default) if machine else default
    if verbose:
        print(f"launch config rows={rows} ncols={ncols} on {machine or '<unknown gpu>'}: {cfg}")
    return cfg


def launch_for(cfg) -> object | None:
    """The C ABI launch struct for a `(block, num_warps)` pair (None: library default)."""
    if cfg is None:
        return None
    _block, warps = cfg
    if not warps:
        return None
    if warps <= 1:
        return launch_struct(VARIANT_WARP_ROW, 0, 0)
    if warps >= 32:
        return launch_struct(VARIANT_CLUSTER, 0, 0, 0)
    return launch_struct(VARIANT_CTA_ROW, 32 * int(warps), 0)


# ---------------------------------------------------------------- the choice rule
@dataclasses.dataclass
class Result:
    block: int
    num_warps: int
    ms: float

    def __str__(self) -> str:
        return f"block={self.block:6d} num_warps={self.num_warps:2d} {self.ms:8.4f} ms"


def best_of(results: list) -> list:
    ok = [r for r in results if math.isfinite(r.ms)]
    if not ok:
        raise RuntimeError(f"no candidate launch configuration could be measured ({len(results)} tried)")
    return sorted(ok, key=lambda r: r.ms)


def choose(results: list, default: tuple, noise: float = NOISE) -> tuple:
    """Keep `default` unless the fastest candidate beats it by more than `noise`."""
    ranked = best_of(results)
    best = ranked[0]
    fix = next((r for r in results if (r.block, r.num_warps) == tuple(default)), None)
    if fix is None or best.ms <= 0:
        return tuple(default), float("nan"), "the default was not measurable: keeping it"
    gain = fix.ms / best.ms
    if gain <= 1.0 + noise:
        return tuple(default), gain, f"within noise ({gain:.2f}x): keeping the default"
    return (best.block, best.num_warps), gain, f"{gain:.2f}x better than the default"


def parameter_identity(params: dict | None) -> tuple:
    """Exact identity of binary64 scalars (hex), as neptune_codegen/autotune.py:392-394."""
    return tuple((key, float(value).hex()) for key, value in sorted((params or {}).items()))


def parameter_tag(params: dict | None) -> str:
    """Identifier-safe exact tag of the parameters (same scheme as autotune.py:397-418)."""
    identity = parameter_identity(params)
    tags = []
    for key, exact in identity:
        value = float.fromhex(exact)
        short = f"{value:g}"
        tag = short.replace(".", "p").replace("-", "m").replace("+", "a")
        if not math.isfinite(value) or float(short).hex() != exact:
            tag += "_h" + exact.replace("-", "m").replace("+", "a").replace(".", "p")
        tags.append("_" + key + tag)
    if len(identity) > 1 or any(not key.isalpha() for key, _ in identity):
        tags.append("_h" + hashlib.sha256(repr(identity).encode()).hexdigest()[:16])
    return "".join(tags)


def op_key(lib: str, name: str, params: dict | None, keepdim: bool,
           block: int | None = None, num_warps: int | None = None) -> str:
    """Registered op name: parameters, output rank and launch configuration (autotune.py:421-432)."""
    tag = "_keep" if keepdim else ""
    tag += parameter_tag(params)
    if block is not None or num_warps is not None:
        tag += f"_b{block}w{num_warps}"
    return f"{lib}::{name}{tag}"


def search(name: str, rows: int, ncols: int, dtype=None, device: str = "cuda", reps: int = 50,
           candidates=CANDIDATES, params: dict | None = None, warmup: int = 5, rounds: int = 3) -> list:
    """Time every candidate through the C ABI with CUDA events; fastest first.

    Each round replays `reps` launches captured in one CUDA graph, so a small shape measures device
    time rather than the Python launch path (a candidate that cannot be captured is timed eagerly)."""
    import torch

    from neptune_opt_b200 import template

    if dtype is None:
        dtype = torch.float32
    x = torch.randn(rows, ncols, device=device, dtype=dtype).abs().contiguous()
    out = torch.empty(rows, device=device, dtype=dtype)
    results = []
    for block, warps in candidates:
        def launch(block=block, warps=warps):
            template.launch_reduction(name, "serial", x, out, rows, ncols, block, warps, params)

        try:
            for _ in range(warmup):
                launch()
            torch.cuda.synchronize()
        except Exception as exc:  # noqa: BLE001
            results.append(Result(block, warps, float("inf")))
            print(f"      block={block} num_warps={warps} cannot launch: {type(exc).__name__}: {exc}")
            continue
        run = None
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    launch()
            run = graph.replay
        except Exception:  # noqa: BLE001
            torch.cuda.synchronize()

            def run(launch=launch):
                for _ in range(reps):
                    launch()
        times = []
        for _ in range(rounds):
            run()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            run()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end) / reps)
        results.append(Result(block, warps, min(times)))
    return best_of(results)


def choose_many(per_shape: list, default: tuple = DEFAULT, noise: float = NOISE) -> tuple:
    """One configuration for a bucket measured at several shapes: the candidate whose WORST gain
    over the default across the shapes is largest (the rule of neptune_codegen/autotune.py:297-356),
    kept only if that worst case clears `noise`. `per_shape` is a list of measured candidate lists.
    Returns `(config, worst_case_gain, reason)`."""
    runs = []
    for results in per_shape:
        ms = {(r.block, r.num_warps): r.ms for r in results if math.isfinite(r.ms) and r.ms > 0}
        if tuple(default) in ms:
            runs.append(ms)
    if not runs:
        return tuple(default), float("nan"), "the default was not measurable: keeping it"
    shared = set.intersection(*(set(run) for run in runs))
    scored = sorted(((min(run[tuple(default)] / run[cfg] for run in runs), cfg) for cfg in shared),
                    key=lambda item: (-item[0], item[1]))
    worst, cfg = scored[0]
    if cfg == tuple(default) or worst <= 1.0 + noise:
        return tuple(default), worst, f"within noise ({worst:.2f}x worst case): keeping the default"
    return cfg, worst, f"{worst:.2f}x better than the default in the worst case"


def measure_shapes(name: str, shapes, dtype=None, device: str = "cuda", reps: int = 50,
                   candidates=CANDIDATES, rounds: int = 3, params: dict | None = None,
                   log=print) -> tuple:
    """Time every candidate at every `(rows, ncols)` shape and reduce each bucket to one choice
    (neptune_codegen/autotune.py:512-548). Returns `(table, records)`: `table` maps shape keys to
    configurations and holds only deviations from the default; `records` keeps each shape's
    measurements."""
    per_bucket, records = {}, []
    for rows, ncols in shapes:
        key = shape_key(rows, ncols)
        results = search(name, rows, ncols, dtype=dtype, device=device, reps=reps, candidates=candidates,
                         params=params, rounds=rounds)
        picked, gain, why = choose(results, DEFAULT)
        log(f"  rows={rows:6d} ncols={ncols:7d} {key}: " + ", ".join(str(r) for r in results[:3]) +
            f" -> {picked} ({why})")
        records.append({"shape": (rows, ncols), "key": key, "picked": picked, "gain": gain,
                        "results": [(r.block, r.num_warps, r.ms) for r in results]})
        per_bucket.setdefault(key, []).append(results)
    out = {}
    for key, runs in sorted(per_bucket.items()):
        cfg, worst, why = choose_many(runs, DEFAULT)
        log(f"  bucket {key} ({len(runs)} shape(s)) -> {cfg}: {why}")
        if cfg != DEFAULT:
            out[key] = cfg
    return out, records


def merge_table(all_tables: dict, machine: str, measured_on: str, body: dict, noise: float = NOISE) -> dict:
    """`all_tables` with `machine`'s entry replaced by a fresh measurement (other machines kept)."""
    merged = {m: dict(entry) for m, entry in all_tables.items()}
    merged[machine] = {"measured_on": measured_on, "noise": noise, "table": _valid(body)}
    return merged


def render_tables(all_tables: dict) -> str:
    """Python source of `launch_table.py` for the given tables (deterministic order)."""
    lines = ['"""Measured launch configurations for the CUDA folds -- only deviations from',
             '`autotune.default_config` are listed, keyed by `(rows class, pow2 width bucket)`.',
             '',
             'Written by `python -m neptune_opt_b200.autotune --write` (autotune.measure_shapes on the',
             'machine named in `measured_on`); a machine without an entry uses the default.',
             '"""',
             "TABLES = {"]
    for machine in sorted(all_tables):
        entry = all_tables[machine]
        lines.append(f"    {machine!r}: {{")
        lines.append(f"        'measured_on': {entry.get('measured_on', '')!r},")
        lines.append(f"        'noise': {float(entry.get('noise', NOISE))!r},")
        lines.append("        'table': {")
        for key, cfg in sorted(_valid(entry.get("table", {})).items()):
            lines.append(f"            {tuple(key)!r}: {tuple(cfg)!r},")
        lines.append("        },")
        lines.append("    },")
    lines.append("}")
    return "\n".join(lines) + "\n"


def write_tables(path: str, all_tables: dict) -> None:
    with open(path, "w") as f:
        f.write(render_tables(all_tables))


# The measurement campaign: every rows class at widths across the buckets the folds serve, each
# bucket at two widths (a power of two and a ragged one) so the bucket's choice is a worst case.
CAMPAIGN_WIDTHS = (256, 1000, 1024, 3000, 4096, 12000, 16384, 50000, 65536, 200000, 262144)
CAMPAIGN_ROWS = (1, 4, 8, 64, 4096)
CAMPAIGN_MAX_ELEMS = 1 << 26


def campaign_shapes() -> list:
    shapes = []
    for ncols in CAMPAIGN_WIDTHS:
        for rows in CAMPAIGN_ROWS:
            shapes.append((max(1, min(rows, CAMPAIGN_MAX_ELEMS // ncols)) if rows > THIN_ROWS else rows, ncols))
    return shapes


def main(argv=None) -> int:
    import argparse
    import os

    ap = argparse.ArgumentParser(description="Measure the CUDA fold launch table on this GPU.")
    ap.add_argument("--skeleton", default="logsumexp")
    ap.add_argument("--dtype", default="float32", choices=("float32", "bfloat16", "float16"))
    ap.add_argument("--write", action="store_true", help="rewrite launch_table.py with this machine's entry")
    ap.add_argument("--reps", type=int, default=50)
    args = ap.parse_args(argv)
    import torch

    name = torch.cuda.get_device_name(torch.cuda.current_device())
    machine = machine_key(name)
    dtype = getattr(torch, args.dtype)
    print(f"measuring {args.skeleton} ({args.dtype}) on {name} -> table '{machine}'")
    body, _ = measure_shapes(args.skeleton, campaign_shapes(), dtype=dtype, reps=args.reps)
    print(f"deviations from the default: {body or 'none'}")
    if args.write:
        merged = merge_table(tables(), machine, f"{name}, {args.skeleton} {args.dtype}", body)
        write_tables(os.path.join(os.path.dirname(os.path.abspath(__file__)), "launch_table.py"), merged)
        print("launch_table.py written")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
