"""Custom-op registration of the CUDA kernels, so rewritten graph regions call them.

Mirrors neptune_codegen/torch_op.py: `as_cuda_op`/`op_handle` register one op per (skeleton, exact
parameters, keepdim, launch configuration, plan) with schema `(Tensor x) -> Tensor`;
`as_state_op`/`state_op_handle` register the structured RMSNorm op `(Tensor x, Tensor gamma) ->
Tensor` and dispatch segment pooling to `as_segment_op`/`segment_op_handle` with schema
`(Tensor data, Tensor segments) -> Tensor`. Every handle is a `torch._ops.OpOverload` whose
fake/meta evaluation computes metadata only.

How a per-key op runs. Its only kernel is a CompositeImplicitAutograd body: it checks the
reference's input contract, then calls the generic C++-registered region op of
libneptune_b200_torch.so (`torch.ops.nb200.fold / rms_norm / segment_pool / softmax`) with the
key's skeleton, parameters, plan and launch baked in as arguments. So
* eager calls run the kernels through that C++ op (which calls the C ABI on the current stream);
* a graph rewritten by the reference (neptune_recognize/rewrite.py:159-217) holds the per-key
  node, which exports, saves and loads like any op;
* when AOTInductor compiles such a graph (neptune_opt/ab.py:145-172), tracing replaces the per-key
  node by its body, so the package calls only `nb200::*` ops by name and runs without Python --
  the reference instead embeds its generated Triton kernels in the package.

Differences from the reference, by design:
* the ops are composite ops over C++ ops instead of `triton_op`s; `as_triton_op`,
  `triton_op_name` and `_TRITON_OPS` remain as aliases of the CUDA names so the reference's
  callers keep working;
* descriptor validation of segment pooling never traps the GPU: the kernels OR violations into a
  sticky per-device status word (one word per device, shared by every launch path) and malformed
  spans pool to NaN (as the reference kernel itself does). `segment_status()` reads and clears the
  word; with NEPTUNE_B200_SYNC_CHECKS=1 every eager call checks it and raises the reference's
  RuntimeError messages.
"""
from __future__ import annotations

import ctypes
import math
import os
import struct

from neptune_opt_b200 import _lib, autotune
from neptune_opt_b200.skeletons import SKELETONS, checked_params, param_defaults
from neptune_opt_b200.template import (_on_device, _ptr, _row_last_layout, _validate_row_last,
                                       current_stream, dtype_code, launch_reduction, launch_rms_norm,
                                       split_launch_shape, validate_plan, validate_rms_inputs)

_CUDA_OPS: dict[str, object] = {}
_TRITON_OPS = _CUDA_OPS  # the reference's registry name
_FRAGMENTS: dict[str, object] = {}


def _nb200():
    """torch.ops.nb200 with the C++ region ops registered (libneptune_b200_torch.so)."""
    import torch

    from neptune_opt_b200 import aot

    aot.load()
    return torch.ops.nb200


def _tracing(*tensors) -> bool:
    """True while fake, meta or functional tensors trace the op (export, AOTInductor, FakeTensorMode)."""
    from torch._subclasses.fake_tensor import FakeTensor
    from torch.utils._python_dispatch import is_traceable_wrapper_subclass

    return any(isinstance(t, FakeTensor) or t.device.type == "meta" or is_traceable_wrapper_subclass(t)
               for t in tensors)


def _register(op_name: str, schema: str, body):
    """Define `lib::name` with `schema`; its one kernel is the CompositeImplicitAutograd `body`."""
    import torch

    lib, name = op_name.split("::", 1)
    frag = _FRAGMENTS.get(lib)
    if frag is None:
        frag = _FRAGMENTS[lib] = torch.library.Library(lib, "FRAGMENT")
    frag.define(name + schema)
    frag.impl(name, body, "CompositeImplicitAutograd")
    return _overload(lib, op_name)


def _overload(lib: str, op_name: str):
    import torch

    packet = getattr(getattr(torch.ops, lib), op_name.split("::", 1)[1])
    return getattr(packet, "default", packet)


# ---------------------------------------------------------------- scalar skeleton ops
def as_cuda_op(name: str, block: int | None = None, num_warps: int | None = None, lib: str = "neptune",
               params: dict | None = None, keepdim: bool = False, plan: str = "serial"):
    """Register (once) and return the op for one fold (torch_op.py:16-114)."""
    validate_plan(plan)
    if name not in SKELETONS:
        raise KeyError(f"unknown skeleton {name!r}; have {sorted(SKELETONS)}")
    if plan == "split":
        block = autotune.SPLIT_BLOCK if block is None else block
        num_warps = 8 if num_warps is None else num_warps
        if SKELETONS[name].two_pass:
            raise NotImplementedError("two_pass needs extended carried state; pair merge refused")
    values = checked_params(name, {**param_defaults(name), **(params or {})})
    key = autotune.op_key(lib, name, {k: values[k] for k in sorted(values)}, keepdim, block, num_warps)
    if plan != "serial":
        key += "_plan_split"
    if key in _CUDA_OPS:
        return _CUDA_OPS[key]

    from neptune_opt_b200.aot import fold_params

    sk_id = SKELETONS[name].id
    fparams = fold_params(name, values)
    plan_code = 0 if plan == "serial" else 1

    def _body(x):
        _validate_row_last(x, metadata=_tracing(x))
        cfg = (block, num_warps)
        if plan == "split":
            split_launch_shape(x.shape[-1], block)
        elif block is None or num_warps is None:
            shape = tuple(x.shape)
            concrete = all(type(d) is int for d in shape)
            rows = math.prod(shape[:-1]) if concrete else None
            chosen = (autotune.best_config(rows, shape[-1], x.dtype, x.device) if concrete
                      else autotune.DEFAULT)
            cfg = (chosen[0] if block is None else block, chosen[1] if num_warps is None else num_warps)
        return _nb200().fold(x, sk_id, fparams, keepdim, plan_code, int(cfg[0] or 0), int(cfg[1] or 0))

    op = _register(key, "(Tensor x) -> Tensor", _body)
    _CUDA_OPS[key] = op
    return op


as_triton_op = as_cuda_op


def op_handle(name: str, params: dict | None = None, lib: str = "neptune", keepdim: bool = False,
              block: int | None = None, num_warps: int | None = None, plan: str = "serial"):
    """The OpOverload for a compiled skeleton, for building graph nodes (torch_op.py:117-134)."""
    return as_cuda_op(name, block=block, num_warps=num_warps, params=params, lib=lib, keepdim=keepdim, plan=plan)


def cuda_op_name(name: str, lib: str = "neptune") -> str:
    return f"{lib}.{name}"


triton_op_name = cuda_op_name


# ---------------------------------------------------------------- softmax-family ops
_READOUT_OPS: dict[tuple, object] = {}


def softmax_op_handle(log: bool = False, lib: str = "neptune"):
    """OpOverload `(Tensor x) -> Tensor` of the fused softmax (log=False) / log_softmax readout."""
    key = (lib, bool(log))
    if key not in _READOUT_OPS:
        mode = 1 if log else 0

        def _body(x):
            _validate_row_last(x, metadata=_tracing(x))
            return _nb200().softmax(x, mode)[0]

        _READOUT_OPS[key] = _register(f"{lib}::{'log_softmax' if log else 'softmax'}_lastdim", "(Tensor x) -> Tensor",
                                      _body)
    return _READOUT_OPS[key]


# ---------------------------------------------------------------- structured RMSNorm
_STATE_OPS: dict[tuple, object] = {}


def as_state_op(name, params=None, plan="serial", lib="neptune"):
    """Structured two-input op (torch_op.py:145-190); segments dispatch to `as_segment_op`."""
    if name in ("segment_sum", "segment_mean"):
        return as_segment_op(name, params=params, plan=plan, lib=lib)
    if name != "rms_norm":
        raise KeyError(f"unknown structured reduction {name!r}")
    validate_plan(plan)
    params = dict(params or {})
    eps = params.get("eps")
    if params.keys() != {"eps"} or type(eps) not in (int, float) or not math.isfinite(eps) or eps <= 0:
        raise ValueError("RMSNorm requires only the explicit eps parameter")
    key = (lib, "rms_norm", autotune.parameter_identity(params), plan)
    if key in _STATE_OPS:
        return _STATE_OPS[key]
    impl_name = f"state_rms_norm{autotune.parameter_tag(params)}_plan_{plan}"
    eps_value = float(eps)

    def _body(x, gamma):
        validate_rms_inputs(x, gamma, params, plan=plan, metadata=_tracing(x, gamma))
        return _nb200().rms_norm(x, gamma, eps_value)

    op = _register(f"{lib}::{impl_name}", "(Tensor x, Tensor gamma) -> Tensor", _body)
    _STATE_OPS[key] = op
    return op


def state_op_handle(name, params=None, plan="serial", lib="neptune"):
    return as_state_op(name, params=params, plan=plan, lib=lib)


# ---------------------------------------------------------------- ordered segment pooling
_SEGMENT_OPS: dict[tuple, object] = {}

SPAN_MESSAGES = (
    (1, "segment lengths must be nonnegative and within data bounds"),
    (2, "segment lengths must sum to data axis0 size"),
    (4, "segment boundaries out of data bounds"),
    (8, "segment boundaries must be monotonic"),
)


def _segment_params(name, params=None, plan="serial"):
    """Parameter contract of torch_op.py:208-232."""
    if name not in ("segment_sum", "segment_mean"):
        raise KeyError(f"unknown segment reduction {name!r}")
    validate_plan(plan)
    if plan != "serial":
        raise NotImplementedError("segment split cannot preserve ordered storage-dtype rounding; use serial")
    params = dict(params or {})
    unknown = params.keys() - {"initial", "offsets", "unsafe"}
    if unknown:
        raise ValueError(f"unknown segment parameters: {sorted(unknown)}")
    initial = params.get("initial")
    if initial is not None:
        if isinstance(initial, bool) or not isinstance(initial, (int, float)):
            raise TypeError("segment initial must be a finite Python scalar or None")
        initial = float(initial)
        if not math.isfinite(initial):
            raise ValueError("segment initial must be finite")
    offsets, unsafe = params.get("offsets", False), params.get("unsafe", False)
    if type(offsets) is not bool or type(unsafe) is not bool:
        raise TypeError("segment offsets and unsafe must be bool")
    return {"initial": initial, "offsets": offsets, "unsafe": unsafe}


def _initial_bits(initial) -> int:
    """fp32 bit pattern of `initial` (fp32 conversion first, as native CUDA scalar conversion)."""
    value = 0.0 if initial is None else initial
    try:
        value = struct.unpack("f", struct.pack("f", value))[0]
    except OverflowError:
        value = float("-inf") if value < 0 else float("inf")
    return struct.unpack("I", struct.pack("f", value))[0]


def validate_segment_inputs(data, segments, *, metadata=False, offsets=False, initial=None, unsafe=False,
                            reduce="sum", plan="serial"):
    """Metadata-only contract (torch_op.py:340-367); returns the output shape."""
    import torch

    _segment_params("segment_" + reduce, {"initial": initial, "offsets": offsets, "unsafe": unsafe}, plan)
    if data.layout != torch.strided or segments.layout != torch.strided:
        raise TypeError("segment requires strided data and segments")
    if data.ndim < 1 or segments.ndim != 1:
        raise ValueError("segment data rank must be >= 1 and segments rank must be 1")
    if data.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("segment data dtype must be float16/bfloat16/float32")
    if initial is not None and abs(initial) > torch.finfo(data.dtype).max:
        raise RuntimeError("segment initial cannot be converted to input dtype without overflow")
    if segments.dtype not in (torch.int32, torch.int64):
        raise TypeError("segment index dtype must be int32/int64")
    if data.device != segments.device:
        raise ValueError("segment tensors must be on the same device")
    if not metadata and data.device.type != "cuda":
        raise ValueError("segment execution requires CUDA device")
    if offsets:
        torch._check(segments.shape[0] >= 1, lambda: "segment offsets needs at least one boundary")
    count = segments.shape[0] - 1 if offsets else segments.shape[0]
    return (count,) + data.shape[1:]


def _sync_checks() -> bool:
    return os.environ.get("NEPTUNE_B200_SYNC_CHECKS", "") not in ("", "0")


def segment_status_word(device):
    """The device's sticky descriptor-status word (int32, zero until a violation is recorded). It is
    the word the C++ region ops use too, so every launch path records into one word per device."""
    import torch

    index = device.index if device.index is not None else torch.cuda.current_device()
    return _nb200().segment_status_word(index)


def segment_status(device=None, clear: bool = True) -> int:
    """Read (and by default clear) the descriptor-status bits recorded on `device` since the last
    clear: 1 length negative or > nrows, 2 lengths do not cover nrows, 4 boundary out of
    [0, nrows], 8 boundaries decreasing. Synchronises with the device."""
    import torch

    word = segment_status_word(torch.device("cuda", torch.cuda.current_device()) if device is None else device)
    bits = int(word.item())
    if clear and bits:
        word.zero_()
    return bits


def check_segment_status(status) -> None:
    """Raise the reference's RuntimeError for the first violated descriptor condition."""
    bits = int(status.item()) if hasattr(status, "item") else int(status)
    for bit, message in SPAN_MESSAGES:
        if bits & bit:
            raise RuntimeError(message)


def _index_code(t) -> int:
    return _lib.INDEX_CODES[str(t.dtype).removeprefix("torch.")]


def _segment_bounds(data, segments, *, offsets, unsafe, status):
    """(bounds tensor, index code, element stride) for the pooling kernel.

    Offsets are read by the pooling kernel as they are (any int32/int64 stride), which also validates
    them. Lengths become int64 spans cat(0, cumsum(lengths)) in one kernel that validates them
    (torch_op.py:370-387)."""
    import torch

    if offsets:
        return segments, _index_code(segments), segments.stride(0) if segments.numel() else 1
    nseg = segments.shape[0]
    spans = torch.empty(nseg + 1, dtype=torch.int64, device=data.device)
    lib = _lib.load()
    with _on_device(data.device):
        rc = lib.nb200_segment_spans(_ptr(segments), _index_code(segments), nseg,
                                     segments.stride(0) if segments.numel() else 1, int(unsafe), data.shape[0],
                                     _ptr(spans), _ptr(status), ctypes.c_void_p(current_stream(data.device)))
    _lib.check(rc, "neptune segment spans")
    return spans, _lib.INDEX_CODES["int64"], 1


def _launch_segment(name, data, segments, params, plan):
    """torch_op.py:390-410: boundaries, fresh output, one pooling launch (plus one span launch for
    lengths)."""
    import torch

    shape = validate_segment_inputs(data, segments, reduce=name.removeprefix("segment_"), plan=plan, **params)
    status = segment_status_word(data.device)
    bounds, idx, bstride = _segment_bounds(data, segments, offsets=params["offsets"], unsafe=params["unsafe"],
                                           status=status)
    channels = 1
    for size in data.shape[1:]:
        channels = channels * size
    out = torch.empty(shape, dtype=data.dtype, device=data.device)
    if not ((type(shape[0]) is int and shape[0] == 0) or (type(channels) is int and channels == 0)):
        flat = data.reshape(data.shape[0], channels)
        lib = _lib.load()
        initial = params["initial"]
        with _on_device(data.device):
            rc = lib.nb200_segment_pool(_ptr(flat), dtype_code(data.dtype), data.shape[0], channels,
                                        flat.stride(0), flat.stride(1), _ptr(bounds), idx, bstride, shape[0],
                                        1 if name == "segment_mean" else 0, int(initial is not None),
                                        _initial_bits(initial), _ptr(out), _ptr(status),
                                        ctypes.c_void_p(current_stream(data.device)))
        _lib.check(rc, f"neptune {name}")
    if _sync_checks():
        check_segment_status(segment_status(data.device))
    return out


def run_segment_pool(data, segments, *, reduce="sum", offsets=False, initial=None, unsafe=False, plan="serial"):
    """Direct launch (torch_op.py:413-424); Fake/meta calls return metadata only."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensor

    name = "segment_" + reduce
    params = _segment_params(name, {"initial": initial, "offsets": offsets, "unsafe": unsafe}, plan)
    if data.device.type == "meta" or isinstance(data, FakeTensor):
        shape = validate_segment_inputs(data, segments, metadata=True, reduce=reduce, plan=plan, **params)
        return torch.empty(shape, dtype=data.dtype, device=data.device)
    return _launch_segment(name, data, segments, params, plan)


def as_segment_op(name, params=None, plan="serial", lib="neptune"):
    """Two-tensor op (torch_op.py:427-457); constants live in the op's identity."""
    params = _segment_params(name, params, plan)
    numeric = {k: v for k, v in params.items() if v is not None}
    identity = (lib, name, params["initial"] is None, autotune.parameter_identity(numeric), plan)
    if identity in _SEGMENT_OPS:
        return _SEGMENT_OPS[identity]
    import hashlib

    impl_name = f"{name}_serial_h" + hashlib.sha256(repr(identity[1:]).encode()).hexdigest()[-10:]

    reduce_code = 1 if name == "segment_mean" else 0
    reduce = name.removeprefix("segment_")

    def _body(data, segments):
        tracing = _tracing(data, segments)
        validate_segment_inputs(data, segments, metadata=tracing, reduce=reduce, plan=plan, **params)
        out = _nb200().segment_pool(data, segments, params["offsets"], reduce_code, params["initial"],
                                    params["unsafe"])
        if not tracing and _sync_checks():
            check_segment_status(segment_status(data.device))
        return out

    op = _register(f"{lib}::{impl_name}", "(Tensor data, Tensor segments) -> Tensor", _body)
    _SEGMENT_OPS[identity] = op
    return op


def segment_op_handle(name, params=None, plan="serial", lib="neptune"):
    return as_segment_op(name, params=params, plan=plan, lib=lib)
