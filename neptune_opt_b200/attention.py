"""Fused single-pass attention on the sm_100a tensor cores (nb200_attention).

O = softmax(scale * Q K^T [+ causal mask]) V per (batch, head) with bf16 Q, K, V, O of shape
[B, H, S, D], fp32 scores and an fp32 online max/sum repair (the exp(c - s) rescale of the
repaired fold applied to attention rows), and optionally the fp32 natural log-sum-exp of each
query row's scaled scores, [B, H, S].

The reference has no attention kernel (its roadmap declares one out of scope); the contract here
follows torch.nn.functional.scaled_dot_product_attention with is_causal (key index <= query
index) and its default scale 1/sqrt(D). Errors follow the backend's convention: TypeError for
dtypes, ValueError for devices, shapes and scale, NotImplementedError for head dimensions the
kernel is not built for.
"""
from __future__ import annotations

import math

from neptune_opt_b200 import _lib
from neptune_opt_b200.template import _on_device, current_stream

HEAD_DIMS = (128,)
OP_NAME = "neptune_b200::attention"


def validate_attention_inputs(q, k, v, scale):
    import torch

    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"attention: {name} must be a tensor")
        if t.dtype != torch.bfloat16:
            raise TypeError(f"attention: {name} must be bfloat16, got {t.dtype}")
        if t.dim() != 4:
            raise ValueError(f"attention: {name} must be [batch, heads, seq, head_dim], got {tuple(t.shape)}")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"attention: q, k, v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if q.device != k.device or q.device != v.device:
        raise ValueError("attention: q, k, v must be on one device")
    if q.device.type != "cuda" and q.device.type != "meta":
        raise ValueError(f"attention: inputs must be CUDA tensors, got {q.device}")
    d = q.shape[-1]
    if d not in HEAD_DIMS:
        raise NotImplementedError(f"attention: head_dim {d} is not supported (built for {HEAD_DIMS})")
    s = 1.0 / math.sqrt(d) if scale is None else float(scale)
    if not (math.isfinite(s) and s > 0.0):
        raise ValueError(f"attention: scale must be finite and positive, got {scale}")
    return s


def launch_attention(q, k, v, o, lse, *, causal: bool, scale: float) -> None:
    """One nb200_attention call on the current stream of q's device (all tensors contiguous)."""
    lib = _lib.load()
    b, h, s, d = q.shape
    with _on_device(q.device):
        rc = lib.nb200_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                 lse.data_ptr() if lse is not None else None, b, h, s, d, 1 if causal else 0,
                                 scale, current_stream(q.device))
    _lib.check(rc, "nb200_attention")


def run_attention(q, k, v, *, causal: bool = False, scale=None, return_lse: bool = False):
    """Fresh O (and LSE when asked) for contiguous copies of q, k, v."""
    import torch

    sc = validate_attention_inputs(q, k, v, scale)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:-1], device=q.device, dtype=torch.float32) if return_lse else None
    if q.device.type != "meta" and q.numel():
        launch_attention(q, k, v, o, lse, causal=causal, scale=sc)
    return (o, lse) if return_lse else o


_OP = None


def attention_op():
    """Op `neptune_b200::attention(q, k, v, causal, scale) -> (O, LSE)`. Like the region ops, its one
    kernel is a composite body that checks the contract and calls the C++-registered
    `nb200::attention`, so a graph holding it exports, and AOTInductor packages it as a call of the
    C++ op."""
    global _OP
    if _OP is not None:
        return _OP
    from neptune_opt_b200.torch_op import _nb200, _register

    def _body(q, k, v, causal, scale):
        sc = validate_attention_inputs(q, k, v, scale)
        return tuple(_nb200().attention(q, k, v, causal, sc))

    _OP = _register(OP_NAME, "(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> (Tensor, Tensor)", _body)
    return _OP
