"""Runtime contracts and launches of the row-last folds, RMSNorm and the softmax-family readouts.

Mirrors the execution half of the reference's neptune_codegen/template.py -- the same functions
(`split_launch_shape`, `_validate_row_last`, `_row_last_layout`, `launch_reduction`, `run`,
`validate_rms_inputs`, `launch_rms_norm`, `run_rms_norm`), arguments, shapes and exception types --
with every launch going to the sm_100a kernels through the C ABI (include/neptune_b200.h). There is
no code generation step: the skeletons are compiled into libneptune_b200.so.
"""
from __future__ import annotations

import ctypes
import math

from neptune_opt_b200 import _lib
from neptune_opt_b200.skeletons import SKELETONS, checked_params, param_defaults

MAX_SPLIT_PARTS = 4096
RMS_SERIAL_MAX_WIDTH = 32768


def validate_plan(plan: str) -> None:
    if plan not in ("serial", "split"):
        raise ValueError(f"unknown reduction plan {plan!r}; expected 'serial' or 'split'")


def split_launch_shape(ncols, block: int) -> tuple:
    """(nparts, next power of two >= nparts); refuses unknown width and capacity overflow
    (neptune_codegen/template.py:114-125)."""
    if type(ncols) is not int:
        raise NotImplementedError("explicit split requires a concrete width; use plan='serial' for dynamic width")
    if type(block) is not int or block <= 0 or block & (block - 1):
        raise ValueError("split BLOCK must be a positive power of two")
    if ncols <= 0:
        raise ValueError("split requires positive width")
    nparts = (ncols + block - 1) // block
    if nparts > MAX_SPLIT_PARTS:
        raise NotImplementedError(f"split needs {nparts} partials, exceeding capacity {MAX_SPLIT_PARTS}; use serial")
    return nparts, 1 << (nparts - 1).bit_length()


def _validate_row_last(x, *, metadata: bool = False):
    """dtype/layout/device/width contract of template.py:338-352."""
    import torch

    if x.layout != torch.strided:
        raise TypeError("Neptune requires a strided tensor")
    if x.ndim < 1:
        raise ValueError("Neptune row-last reductions require rank >= 1")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported Neptune dtype {x.dtype}; expected float16/bfloat16/float32")
    if not metadata and x.device.type != "cuda":
        raise ValueError(f"unsupported Neptune device {x.device}; execution requires CUDA")
    torch._check(x.shape[-1] > 0, lambda: "Neptune requires positive last-dimension width")


def _row_last_layout(x):
    """Flatten only leading dimensions; reshape copies exactly when a view is impossible."""
    rows = 1
    for size in x.shape[:-1]:
        rows = rows * size
    ncols = x.shape[-1]
    return x.reshape(rows, ncols), rows, ncols


def _is_metadata(x) -> bool:
    from torch._subclasses.fake_tensor import FakeTensor

    return isinstance(x, FakeTensor) or x.device.type == "meta"


_DTYPE_CODES: dict = {}


def dtype_code(dtype) -> int:
    code = _DTYPE_CODES.get(dtype)
    if code is None:
        code = _lib.DTYPE_CODES[str(dtype).removeprefix("torch.")]
        _DTYPE_CODES[dtype] = code
    return code


def current_stream(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


class _NoGuard:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_GUARD = _NoGuard()


def _on_device(device):
    """Make `device` current for a launch (its stream belongs to it); free when it already is."""
    import torch

    if device.index is None or device.index == torch.cuda.current_device():
        return _NO_GUARD
    return torch.cuda.device(device.index)


def _ptr(t) -> int:
    return t.data_ptr()


def launch_reduction(name, plan, x2, out, rows, ncols, block=None, num_warps=None, params=None):
    """Launch the fold of skeleton `name` over x2[rows, ncols] into out (contiguous, x's dtype).

    Serial: one C ABI call (nb200_fold). Split: chunk states go to torch-allocated scratch and are
    merged in ascending chunk order (nb200_fold_split). Mirrors template.py:368-390.
    """
    import torch

    from neptune_opt_b200 import autotune

    validate_plan(plan)
    lib = _lib.load()
    values = checked_params(name, params)
    sk = SKELETONS[name]
    p = _lib.params_struct(values)
    with _on_device(x2.device):
        stream = ctypes.c_void_p(current_stream(x2.device))
        if plan == "serial":
            cfg = (block, num_warps) if num_warps is not None else None
            launch = autotune.launch_for(cfg)
            rc = lib.nb200_fold(sk.id, ctypes.byref(p), _ptr(x2), dtype_code(x2.dtype), rows, ncols,
                                x2.stride(0), x2.stride(1), _ptr(out),
                                ctypes.byref(launch) if launch is not None else None, stream)
            _lib.check(rc, f"neptune {name}")
            return
        if sk.two_pass:
            raise NotImplementedError("two_pass needs extended carried state; split refused")
        block = autotune.SPLIT_BLOCK if block is None else block
        nparts, _ = split_launch_shape(ncols, block)
        nbytes = int(lib.nb200_fold_split_scratch_bytes(rows, nparts))
        scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x2.device)
        rc = lib.nb200_fold_split(sk.id, ctypes.byref(p), _ptr(x2), dtype_code(x2.dtype), rows, ncols,
                                  x2.stride(0), x2.stride(1), block, _ptr(scratch), scratch.numel(),
                                  _ptr(out), None, stream)
        _lib.check(rc, f"neptune {name} (split)")


def run(name: str, x, block: int | None = None, num_warps: int | None = None,
        keepdim: bool = False, plan: str = "serial", **params):
    """Execute a skeleton's fold over the last dimension (template.py:393-442).

    Rank >= 1 returns x.shape[:-1] (keepdim appends a singleton), in x's dtype. CUDA float16/
    bfloat16/float32 execute; Fake/meta tensors return metadata only.
    """
    import torch

    from neptune_opt_b200 import autotune

    metadata = _is_metadata(x)
    _validate_row_last(x, metadata=metadata)
    if name not in SKELETONS:
        raise KeyError(f"unknown skeleton {name!r}; have {sorted(SKELETONS)}")
    values = checked_params(name, {**param_defaults(name), **(params or {})})
    validate_plan(plan)
    if plan == "split":
        if SKELETONS[name].two_pass:
            raise NotImplementedError("two_pass needs extended carried state; pair merge refused")
        block = autotune.SPLIT_BLOCK if block is None else block
        split_launch_shape(x.shape[-1], block)
    shape = x.shape[:-1] + ((1,) if keepdim else ())
    out = torch.empty(shape, device=x.device, dtype=x.dtype)
    if metadata:
        return out
    x2, rows, ncols = _row_last_layout(x)
    if isinstance(rows, int) and rows == 0:
        return out
    if plan == "serial" and (block is None or num_warps is None):
        cfg = autotune.best_config(rows, ncols, x.dtype, x.device)
        block = cfg[0] if block is None else block
        num_warps = cfg[1] if num_warps is None else num_warps
    launch_reduction(name, plan, x2, out, rows, ncols, block, num_warps, values)
    return out


# ---------------------------------------------------------------- softmax-family readouts
def run_softmax(x, *, log: bool = False):
    """softmax (log=False) or log_softmax (log=True) over the last dimension in one pass.

    Fresh contiguous output in x's dtype. A row holding NaN or +inf, or no finite element, reads
    out as NaN, as the reference's log_softmax lowering does (neptune_recognize/lowering.py:91-99).
    """
    import torch

    metadata = _is_metadata(x)
    _validate_row_last(x, metadata=metadata)
    y = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    if metadata or x.numel() == 0:
        return y
    x2, rows, ncols = _row_last_layout(x)
    lib = _lib.load()
    with _on_device(x.device):
        rc = lib.nb200_softmax(1 if log else 0, _ptr(x2), dtype_code(x.dtype), rows, ncols, x2.stride(0),
                               x2.stride(1), _ptr(y), None, None, ctypes.c_void_p(current_stream(x.device)))
    _lib.check(rc, "neptune softmax")
    return y


def run_softmax_lse(x, *, log: bool = False):
    """(softmax or log_softmax, logsumexp) from one pass over x."""
    import torch

    metadata = _is_metadata(x)
    _validate_row_last(x, metadata=metadata)
    y = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    lse = torch.empty(x.shape[:-1], device=x.device, dtype=x.dtype)
    if metadata or x.numel() == 0:
        return y, lse
    x2, rows, ncols = _row_last_layout(x)
    lib = _lib.load()
    with _on_device(x.device):
        rc = lib.nb200_softmax(1 if log else 0, _ptr(x2), dtype_code(x.dtype), rows, ncols, x2.stride(0),
                               x2.stride(1), _ptr(y), _ptr(lse), None, ctypes.c_void_p(current_stream(x.device)))
    _lib.check(rc, "neptune softmax")
    return y, lse


def run_l2_normalize(x):
    """(x / norm, norm) with norm = stable_l2 over the last dimension, both in x's dtype."""
    import torch

    metadata = _is_metadata(x)
    _validate_row_last(x, metadata=metadata)
    y = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    norm = torch.empty(x.shape[:-1], device=x.device, dtype=x.dtype)
    if metadata or x.numel() == 0:
        return y, norm
    x2, rows, ncols = _row_last_layout(x)
    lib = _lib.load()
    with _on_device(x.device):
        rc = lib.nb200_l2_normalize(_ptr(x2), dtype_code(x.dtype), rows, ncols, x2.stride(0), x2.stride(1),
                                    _ptr(y), _ptr(norm), None, ctypes.c_void_p(current_stream(x.device)))
    _lib.check(rc, "neptune l2_normalize")
    return y, norm


# ---------------------------------------------------------------- RMSNorm
def validate_rms_inputs(x, gamma, params=None, *, plan="serial", metadata=False):
    """Full-vector RMSNorm contract of template.py:267-291; returns the output shape."""
    import torch

    validate_plan(plan)
    _validate_row_last(x, metadata=metadata)
    params = dict(params or {})
    eps = params.get("eps")
    if params.keys() != {"eps"} or type(eps) not in (int, float) or not math.isfinite(eps) or eps <= 0:
        raise ValueError("RMSNorm requires an explicit finite positive eps")
    if gamma.layout != torch.strided or gamma.ndim != 1:
        raise ValueError("RMSNorm gamma must be a strided 1D tensor")
    if gamma.dtype != x.dtype or gamma.device != x.device:
        raise ValueError("RMSNorm gamma dtype/device must match input")
    torch._check(gamma.shape[0] == x.shape[-1], lambda: "RMSNorm gamma width must match input")
    if type(x.shape[-1]) is not int:
        raise NotImplementedError("RMSNorm first backend requires a static feature width")
    if plan == "serial" and x.shape[-1] > RMS_SERIAL_MAX_WIDTH:
        raise NotImplementedError("resident RMSNorm width exceeds 32768; request split explicitly")
    if plan == "split":
        split_launch_shape(x.shape[-1], 1024)
    return x.shape


def launch_rms_norm(x, gamma, out, *, eps: float, plan="serial", launch=None):
    """One launch of the RMSNorm kernel (both plans: the CUDA kernel folds any width in one pass
    over resident chunks, so the split plan needs no scratch here)."""
    validate_plan(plan)
    flat, rows, width = _row_last_layout(x)
    if isinstance(rows, int) and rows == 0:
        return
    lib = _lib.load()
    with _on_device(x.device):
        rc = lib.nb200_rms_norm(_ptr(flat), _ptr(gamma), dtype_code(x.dtype), rows, width, flat.stride(0),
                                flat.stride(1), gamma.stride(0), float(eps), _ptr(out),
                                ctypes.byref(launch) if launch is not None else None,
                                ctypes.c_void_p(current_stream(x.device)))
    _lib.check(rc, "neptune rms_norm")


def run_rms_norm_host(x, gamma, *, eps: float = 1e-6, out=None, chunk_rows: int = 0, device=None):
    """RMSNorm of host-resident rows (nb200_rms_norm_host): x [..., ncols] and gamma [ncols] are
    contiguous CPU tensors (pinned memory lets the copies overlap); the rows stream through the GPU
    in chunks with copies in both directions overlapping the kernel. Returns `out` (a pinned CPU
    tensor shaped like x unless given), complete once the device's current stream has been
    synchronised. Results equal run_rms_norm on the same rows moved to the device."""
    import torch

    if x.device.type != "cpu" or gamma.device.type != "cpu" or (out is not None and out.device.type != "cpu"):
        raise ValueError("run_rms_norm_host takes host (CPU) tensors")
    if x.dtype not in (torch.float32, torch.bfloat16, torch.float16) or gamma.dtype != x.dtype:
        raise TypeError("run_rms_norm_host: x and gamma must share a float32/bfloat16/float16 dtype")
    if x.dim() < 1 or gamma.dim() != 1 or gamma.shape[0] != x.shape[-1]:
        raise ValueError("run_rms_norm_host: gamma must be 1-D with x's last-dimension width")
    if not (x.is_contiguous() and gamma.is_contiguous()):
        raise ValueError("run_rms_norm_host: x and gamma must be contiguous")
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    elif out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("run_rms_norm_host: out must be a contiguous tensor shaped like x")
    ncols = x.shape[-1]
    rows = x.numel() // ncols if ncols else 0
    if rows == 0:
        return out
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    lib = _lib.load()
    need = lib.nb200_rms_norm_host_work_bytes(dtype_code(x.dtype), ncols, int(chunk_rows))
    if need < 0:
        raise ValueError("run_rms_norm_host: bad width or chunk size")
    with _on_device(dev):
        work = torch.empty(need, dtype=torch.uint8, device=dev)
        rc = lib.nb200_rms_norm_host(_ptr(x), _ptr(gamma), dtype_code(x.dtype), rows, ncols, float(eps),
                                     _ptr(out), int(chunk_rows), _ptr(work), need,
                                     ctypes.c_void_p(current_stream(dev)))
    _lib.check(rc, "neptune rms_norm_host")
    return out


def run_rms_norm(x, gamma, *, eps: float = 1e-6, plan="serial"):
    """Direct structured execution (template.py:322-335): fresh contiguous output."""
    import torch

    params = {"eps": eps}
    metadata = _is_metadata(x)
    shape = validate_rms_inputs(x, gamma, params, plan=plan, metadata=metadata)
    out = torch.empty(shape, device=x.device, dtype=x.dtype)
    if metadata or x.numel() == 0:
        return out
    launch_rms_norm(x, gamma, out, eps=eps, plan=plan)
    return out
