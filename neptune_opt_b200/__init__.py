"""neptune_opt_b200 -- B200 (sm_100a) backend for neptune-opt's fused dependent-reduction path.

A drop-in replacement for the backend half of the reference package `neptune_codegen`
(emitters/sym_to_triton/template/torch_op/autotune/launch_table). The public names a caller of that
backend uses -- `run`, `op_handle`, `as_triton_op`, `state_op_handle`, `as_state_op`,
`run_rms_norm`, `run_segment_pool`, `split_launch_shape`, `MAX_SPLIT_PARTS`, `param_defaults`,
`supported`, `autotune` -- keep their signatures, result shapes/dtypes and exception types. Under
them, every launch is a hand-written CUDA kernel in libneptune_b200.so reached through the C ABI of
include/neptune_b200.h; there is no Triton and no CPU fallback.

Explicit operator library (as neptune_opt's one-function-per-skeleton surface): `logsumexp(x)`,
`stable_l2(x)`, ... plus the fused readouts `softmax(x)`, `log_softmax(x)`, `l2_normalize(x)`,
`rms_norm(x, gamma, eps)`, `segment_sum/segment_mean(data, segments, ...)` and `attention(q, k, v)`.
"""
from __future__ import annotations

from neptune_opt_b200 import autotune  # noqa: F401
from neptune_opt_b200._lib import BackendUnavailable, LIB_PATH, launch_count, load  # noqa: F401
from neptune_opt_b200.attention import attention_op, run_attention  # noqa: F401
from neptune_opt_b200.skeletons import (SKELETONS, all_registered, op_parameters, param_defaults,  # noqa: F401
                                        supported)
from neptune_opt_b200.template import (MAX_SPLIT_PARTS, launch_reduction, run, run_l2_normalize,  # noqa: F401
                                       run_rms_norm, run_rms_norm_host, run_softmax, run_softmax_lse,
                                       split_launch_shape, validate_plan, validate_rms_inputs)
from neptune_opt_b200.torch_op import (_CUDA_OPS, _TRITON_OPS, as_cuda_op, as_segment_op,  # noqa: F401
                                       as_state_op, as_triton_op, check_segment_status, cuda_op_name,
                                       op_handle, run_segment_pool, segment_op_handle, softmax_op_handle,
                                       segment_status, state_op_handle, triton_op_name,
                                       validate_segment_inputs)

__version__ = "0.1.0"


def _make_op(name):
    def op(x, *, plan="serial", **params):
        missing = [p for p in op_parameters(name) if p not in params]
        if missing:
            raise TypeError(f"neptune_opt.{name}() needs {', '.join(missing)}")
        values = {**param_defaults(name), **params}
        return op_handle(name, params=values or None, plan=plan)(x)

    op.__name__ = op.__qualname__ = name
    op.__doc__ = f"Fused {name} over the last dimension; explicit serial/split CUDA plan."
    return op


for _op_name in supported():
    globals()[_op_name] = _make_op(_op_name)


def softmax(x):
    """Fused single-pass softmax over the last dimension."""
    return run_softmax(x, log=False)


def log_softmax(x):
    """Fused single-pass log_softmax over the last dimension."""
    return run_softmax(x, log=True)


def l2_normalize(x):
    """x / stable_l2(x) over the last dimension, one pass."""
    return run_l2_normalize(x)[0]


def rms_norm(x, gamma, eps: float = 1e-6, plan: str = "serial"):
    return run_rms_norm(x, gamma, eps=eps, plan=plan)


def attention(q, k, v, *, causal: bool = False, scale=None, return_lse: bool = False):
    """softmax(scale * q k^T [+ causal mask]) v over bf16 [batch, heads, seq, 128] tensors."""
    return run_attention(q, k, v, causal=causal, scale=scale, return_lse=return_lse)


def segment_sum(data, segments, *, offsets=False, initial=None, unsafe=False):
    return run_segment_pool(data, segments, reduce="sum", offsets=offsets, initial=initial, unsafe=unsafe)


def segment_mean(data, segments, *, offsets=False, initial=None, unsafe=False):
    return run_segment_pool(data, segments, reduce="mean", offsets=offsets, initial=initial, unsafe=unsafe)


__all__ = [
    "MAX_SPLIT_PARTS", "SKELETONS", "BackendUnavailable", "all_registered", "as_cuda_op", "as_segment_op",
    "attention", "attention_op", "run_attention",
    "as_state_op", "as_triton_op", "autotune", "check_segment_status", "cuda_op_name", "l2_normalize",
    "launch_count", "log_softmax", "op_handle", "op_parameters", "param_defaults", "rms_norm", "run",
    "run_l2_normalize", "run_rms_norm", "run_rms_norm_host", "run_segment_pool", "run_softmax", "run_softmax_lse",
    "segment_mean", "segment_op_handle", "segment_status", "segment_sum", "softmax", "softmax_op_handle",
    "split_launch_shape", "state_op_handle", "supported", "triton_op_name", "validate_rms_inputs",
    "validate_segment_inputs",
] + supported()
