"""ctypes binding of libneptune_b200.so, the C ABI declared in include/neptune_b200.h.

The library is loaded from the package directory (built in-tree by
`make -C neptune_opt_b200/csrc`). There is no fallback: if the library is missing or cannot be
loaded, every execution entry point raises, and nothing computes the result any other way.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libneptune_b200.so")

NB200_OK = 0
NB200_ERR_ARG = -1
NB200_ERR_CAPACITY = -2
NB200_ERR_LAUNCH = -3
NB200_ERR_TIMEOUT = -4
NB200_ERR_UNSUPPORTED = -5

DTYPE_CODES = {"float32": 0, "bfloat16": 1, "float16": 2}
INDEX_CODES = {"int32": 0, "int64": 1}

VARIANT_AUTO, VARIANT_WARP_ROW, VARIANT_CTA_ROW, VARIANT_STREAM, VARIANT_CLUSTER = 0, 1, 2, 3, 4


class NB200Params(ctypes.Structure):
    _fields_ = [("tiny", ctypes.c_double), ("alpha", ctypes.c_double), ("T", ctypes.c_double),
                ("beta", ctypes.c_double), ("N", ctypes.c_double), ("eps", ctypes.c_double)]


class NB200Launch(ctypes.Structure):
    _fields_ = [("variant", ctypes.c_int32), ("threads", ctypes.c_int32),
                ("ctas_per_sm", ctypes.c_int32), ("stages", ctypes.c_int32)]


class NB200State(ctypes.Structure):
    _fields_ = [("m", ctypes.c_float), ("acc", ctypes.c_float), ("seen", ctypes.c_int32),
                ("status", ctypes.c_int32)]


STATE_BYTES = ctypes.sizeof(NB200State)

# Every symbol include/neptune_b200.h declares, with (restype, argtypes).
_vp, _i64, _int, _dbl = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double
SIGNATURES = {
    "nb200_last_error": (ctypes.c_char_p, []),
    "nb200_version": (ctypes.c_char_p, []),
    "nb200_launch_count": (ctypes.c_uint64, []),
    "nb200_stream_fault": (_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "nb200_fold": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _int, _i64, _i64, _i64, _i64, _vp,
                          ctypes.POINTER(NB200Launch), _vp]),
    "nb200_softmax": (_int, [_int, _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, ctypes.POINTER(NB200Launch), _vp]),
    "nb200_l2_normalize": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, ctypes.POINTER(NB200Launch), _vp]),
    "nb200_fold_split_scratch_bytes": (_i64, [_i64, _i64]),
    "nb200_fold_split": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _int, _i64, _i64, _i64, _i64, _i64,
                                _vp, _i64, _vp, ctypes.POINTER(NB200Launch), _vp]),
    "nb200_fold_split_noalloc": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _int, _i64, _i64, _i64, _i64,
                                        _i64, _vp, _vp]),
    "nb200_fold_partial": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _int, _i64, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _vp, ctypes.POINTER(NB200Launch), _vp]),
    "nb200_fold_merge": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _i64, _i64, _i64, _i64, _vp, _int, _vp]),
    "nb200_peer_buffer_bytes": (_i64, [_i64, _i64, _i64]),
    "nb200_peer_init": (_int, [_vp, _i64, _int, _i64, _vp]),
    "nb200_peer_fold": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _int, _i64, _i64, _i64, _i64, _i64, _i64,
                               ctypes.POINTER(ctypes.c_void_p), _int, _int, _vp, _vp, _vp]),
    "nb200_peer_push": (_int, [_vp, _i64, _i64, _i64, ctypes.POINTER(ctypes.c_void_p), _int, _int, _vp, _vp]),
    "nb200_peer_merge": (_int, [_int, ctypes.POINTER(NB200Params), _vp, _i64, _i64, _int, _vp, _int, _vp]),
    "nb200_ipc_handle": (_int, [_vp, _vp, ctypes.POINTER(ctypes.c_int64)]),
    "nb200_ipc_open": (_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "nb200_ipc_close": (_int, [_vp]),
    "nb200_rms_norm": (_int, [_vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _dbl, _vp,
                              ctypes.POINTER(NB200Launch), _vp]),
    "nb200_rms_norm_host_work_bytes": (_i64, [_int, _i64, _i64]),
    "nb200_rms_norm_host": (_int, [_vp, _vp, _int, _i64, _i64, _dbl, _vp, _i64, _vp, _i64, _vp]),
    "nb200_segment_spans": (_int, [_vp, _int, _i64, _i64, _int, _i64, _vp, _vp, _vp]),
    "nb200_segment_pool": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _vp, _int, _i64, _i64, _int, _int,
                                  ctypes.c_uint32, _vp, _vp, _vp]),
    "nb200_attention": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, ctypes.c_float, _vp]),
}

_LOCK = threading.Lock()
_LIB = None
_LOAD_ERROR: str | None = None


class BackendUnavailable(RuntimeError):
    """The CUDA library is not built or cannot be loaded; there is no other backend."""


def load():
    """Load the library once; raise BackendUnavailable (never fall back) when it is missing."""
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not os.path.exists(LIB_PATH):
            _LOAD_ERROR = (f"{LIB_PATH} is not built; run `make -C neptune_opt_b200/csrc` "
                           "(or __graft_entry__.build())")
            raise BackendUnavailable(_LOAD_ERROR)
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as exc:
            _LOAD_ERROR = f"cannot load {LIB_PATH}: {exc}"
            raise BackendUnavailable(_LOAD_ERROR) from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = lib
        return lib


def last_error() -> str:
    return load().nb200_last_error().decode("utf-8", "replace")


def launch_count() -> int:
    """Kernel launches this process issued through the library (its own counter)."""
    return int(load().nb200_launch_count())


def stream_fault() -> int:
    """Read and clear the streaming kernels' fault bits (synchronous; 0 means no wait ran out)."""
    bits = ctypes.c_uint32(0)
    check(load().nb200_stream_fault(ctypes.byref(bits)), "nb200_stream_fault")
    return int(bits.value)


def check(rc: int, what: str) -> None:
    """Map a negative nb200_status to the reference's exception classes."""
    if rc == NB200_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == NB200_ERR_ARG:
        raise ValueError(msg)
    if rc in (NB200_ERR_CAPACITY, NB200_ERR_UNSUPPORTED):
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def params_struct(values: dict | None) -> NB200Params:
    v = dict(values or {})
    return NB200Params(float(v.get("tiny", 0.0)), float(v.get("alpha", 0.0)), float(v.get("T", 1.0)),
                       float(v.get("beta", 1.0)), float(v.get("N", 1.0)), float(v.get("eps", 1.0)))


def launch_struct(variant: int = VARIANT_AUTO, threads: int = 0, ctas_per_sm: int = 0, stages: int = 0) -> NB200Launch:
    return NB200Launch(int(variant), int(threads), int(ctas_per_sm), int(stages))
