"""CPU ORACLE -- test infrastructure only.

A restatement of the reference backend's algorithms (Defyli/neptune-opt, package
neptune_codegen) in plain C (oracle.c, loaded here through ctypes). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and only as the checker or the
timed CPU baseline: the product path in neptune_opt_b200 never imports it.

Every array crossing this wrapper is float32 (values of bf16/fp16 inputs are exact in float32) or
int64; results are float32 values that are exactly representable in the requested storage dtype
when a dtype is given. Parity of this oracle with the reference is pinned by
tests/test_oracle_golden.py against vectors the reference itself produced
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

SKELETON_IDS = {
    "logsumexp": 0, "lse_biased": 1, "lse_scaled": 2, "softcap_lse": 3, "stable_l2": 4,
    "linear_attn": 5, "decay_renorm": 6, "sumsq_div": 7, "rmsnorm_max": 8, "variance": 9, "std": 10,
}
DTYPE_CODES = {"float32": 0, "bfloat16": 1, "float16": 2}


class OParams(ctypes.Structure):
    _fields_ = [("tiny", ctypes.c_double), ("alpha", ctypes.c_double), ("T", ctypes.c_double),
                ("beta", ctypes.c_double), ("N", ctypes.c_double), ("eps", ctypes.c_double)]


STATE_DTYPE = np.dtype([("m", np.float32), ("acc", np.float32), ("seen", np.int32), ("status", np.int32)])

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_stp = np.ctypeslib.ndpointer(STATE_DTYPE, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file; returns its path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(os.path.join(_HERE, "oracle.c")):
            build()
        L = ctypes.CDLL(path)
        L.oracle_fold.argtypes = [_int, ctypes.POINTER(OParams), _f32p, _i64, _i64, _i64, _f32p]
        L.oracle_partial.argtypes = [_int, ctypes.POINTER(OParams), _f32p, _i64, _i64, _i64, _i64, _i64, _stp]
        L.oracle_merge.argtypes = [_int, ctypes.POINTER(OParams), _stp, _i64, _i64, _f32p]
        L.oracle_softmax.argtypes = [_int, _f32p, _i64, _i64, _f32p, _f32p]
        L.oracle_l2_normalize.argtypes = [_f32p, _i64, _i64, _int, _f32p, _f32p]
        L.oracle_rms_norm.argtypes = [_f32p, _f32p, _i64, _i64, ctypes.c_double, _int, _f32p]
        L.oracle_rms_scale.argtypes = [_f32p, _i64, _i64, ctypes.c_double, _f32p]
        L.oracle_segment_spans.argtypes = [_i64p, _i64, _int, _int, _i64, _i64p]
        L.oracle_segment_spans.restype = ctypes.c_uint32
        L.oracle_segment_pool.argtypes = [_f32p, _i64, _i64, _i64p, _i64, _int, _int, ctypes.c_float, _int, _f32p]
        L.oracle_round_array.argtypes = [_f32p, _i64, _int]
        L.oracle_num_threads.restype = _int
        _LIB = L
    return _LIB


def num_threads() -> int:
    """Host threads the oracle's parallel loops use."""
    return int(lib().oracle_num_threads())


def _params(values: dict | None) -> OParams:
    v = dict(values or {})
    return OParams(float(v.get("tiny", 0.0)), float(v.get("alpha", 0.0)), float(v.get("T", 1.0)),
                   float(v.get("beta", 1.0)), float(v.get("N", 1.0)), float(v.get("eps", 1.0)))


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def round_dtype(x, dtype: str) -> np.ndarray:
    """Round-to-nearest-even of float32 values to `dtype` (returned as float32)."""
    out = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().oracle_round_array(out.reshape(-1), out.size, DTYPE_CODES[dtype])
    return out


def fold(name: str, x, params: dict | None = None, block: int = 1024) -> np.ndarray:
    """Serial repaired fold of each row of a 2-D float32 array (fp32 result, not narrowed)."""
    x = _f32(x)
    rows, ncols = x.shape
    out = np.empty(rows, np.float32)
    lib().oracle_fold(SKELETON_IDS[name], ctypes.byref(_params(params)), x, rows, ncols, block, out)
    return out


def partial(name: str, x, params: dict | None, col_begin: int, shard: int, block: int) -> np.ndarray:
    """Chunk states [rows, nparts] of columns [col_begin, col_begin + shard)."""
    x = _f32(x)
    rows, ncols = x.shape
    nparts = -(-shard // block)
    states = np.zeros((rows, nparts), STATE_DTYPE)
    lib().oracle_partial(SKELETON_IDS[name], ctypes.byref(_params(params)), x, rows, ncols, col_begin,
                         shard, block, states)
    return states


def merge(name: str, states: np.ndarray, params: dict | None = None) -> np.ndarray:
    """Left fold of [rows, nparts] states in ascending part order, then the finaliser."""
    states = np.ascontiguousarray(states, dtype=STATE_DTYPE)
    rows, nparts = states.shape
    out = np.empty(rows, np.float32)
    lib().oracle_merge(SKELETON_IDS[name], ctypes.byref(_params(params)), states, rows, nparts, out)
    return out


def softmax(x, log: bool = False):
    """(softmax or log_softmax rows, logsumexp per row), fp32."""
    x = _f32(x)
    rows, ncols = x.shape
    y = np.empty_like(x)
    lse = np.empty(rows, np.float32)
    lib().oracle_softmax(1 if log else 0, x, rows, ncols, y, lse)
    return y, lse


def l2_normalize(x, dtype: str = "float32"):
    """(x / norm rounded to dtype, norm rounded to dtype)."""
    x = _f32(x)
    rows, ncols = x.shape
    y = np.empty_like(x)
    norm = np.empty(rows, np.float32)
    lib().oracle_l2_normalize(x, rows, ncols, DTYPE_CODES[dtype], y, norm)
    return y, norm


def rms_norm(x, gamma, eps: float, dtype: str) -> np.ndarray:
    x, gamma = _f32(x), _f32(gamma)
    rows, ncols = x.shape
    out = np.empty_like(x)
    lib().oracle_rms_norm(x, gamma, rows, ncols, float(eps), DTYPE_CODES[dtype], out)
    return out


def rms_scale(x, eps: float) -> np.ndarray:
    """Per-row fp32 scale rsqrt(mean(x^2) + eps) of the RMSNorm stages (binary64 sum, rounded once)."""
    x = _f32(x)
    rows, ncols = x.shape
    scale = np.empty(rows, np.float32)
    lib().oracle_rms_scale(x, rows, ncols, float(eps), scale)
    return scale


def segment_spans(segments, is_offsets: bool, unsafe: bool, nrows: int):
    """(int64 spans, status bits) from lengths or offsets."""
    seg = np.ascontiguousarray(np.asarray(segments, dtype=np.int64))
    nseg = seg.shape[0] - 1 if is_offsets else seg.shape[0]
    spans = np.zeros(max(nseg, 0) + 1, np.int64)
    if is_offsets and seg.shape[0] == 0:
        raise ValueError("segment offsets needs at least one boundary")
    status = lib().oracle_segment_spans(seg, nseg, int(is_offsets), int(unsafe), nrows, spans)
    return spans, int(status)


def segment_pool(data, spans, reduce: str, initial, dtype: str) -> np.ndarray:
    """Ordered storage-dtype pooling; data is [nrows, channels] float32 of storage values."""
    data = _f32(data)
    data2 = data.reshape(data.shape[0], -1) if data.ndim != 2 else data
    data2 = np.ascontiguousarray(data2)
    spans = np.ascontiguousarray(np.asarray(spans, dtype=np.int64))
    nseg = spans.shape[0] - 1
    nrows, channels = data2.shape
    out = np.empty((nseg, channels), np.float32)
    has = initial is not None
    lib().oracle_segment_pool(data2, nrows, channels, spans, nseg, 1 if reduce == "mean" else 0, int(has),
                              float(initial) if has else 0.0, DTYPE_CODES[dtype], out)
    return out.reshape((nseg,) + data.shape[1:])


def attention(q, k, v, causal=False, scale=None):
    """fp64 O = softmax(scale * q k^T [+ causal mask]) v and the natural log-sum-exp per query row.

    q, k, v: arrays [..., S, D] (values of bf16 tensors, any float dtype). The causal mask keeps
    key index <= query index (torch.nn.functional.scaled_dot_product_attention's is_causal for
    equal query and key lengths); scale defaults to 1/sqrt(D). The reference has no attention
    kernel, so this unfused float64 computation is the checker for the fused one; its agreement
    with torch's own CPU scaled_dot_product_attention is pinned in tests/test_oracle_golden.py.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    d = q.shape[-1]
    sc = 1.0 / np.sqrt(d) if scale is None else float(scale)
    s = np.einsum("...qd,...kd->...qk", q, k) * sc
    if causal:
        n = s.shape[-1]
        s = np.where(np.triu(np.ones((n, n), dtype=bool), 1), -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    tot = e.sum(axis=-1, keepdims=True)
    o = np.einsum("...qk,...kd->...qd", e / tot, v)
    return o, (m + np.log(tot))[..., 0]
