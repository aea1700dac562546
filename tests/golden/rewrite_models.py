"""Small modules, written as a user writes them in eager PyTorch, whose graphs the reference's
front end (neptune_opt.apply -> neptune_recognize.rewrite_match) rewrites into this backend's ops.

Shared by make_rewrites.py (which exports them, runs the reference's apply with this backend bound
in and saves the rewritten programs as fixtures) and by the tests that load and run those
fixtures. Each entry: module class, input builder (seeded; shapes and dtypes of the export),
apply() keyword arguments, and the oracle check of its output.
"""
from __future__ import annotations

import torch


class LogsumexpRows(torch.nn.Module):
    """torch.logsumexp over the last dimension (the reference lowers the compound op)."""

    def forward(self, x):
        return torch.logsumexp(x, dim=-1)


class ShiftedExpSum(torch.nn.Module):
    """The max-shifted sum of exponentials written out, scaled afterwards (a graph boundary)."""

    def forward(self, x):
        top = x.amax(dim=-1, keepdim=True)
        total = torch.exp(x - top).sum(dim=-1, keepdim=True)
        return (top + torch.log(total)).squeeze(-1) * 0.5


class RowL2(torch.nn.Module):
    """Overflow-safe row L2 norm: scale by the largest magnitude before squaring."""

    def forward(self, x):
        big = x.abs().amax(dim=-1, keepdim=True).clamp_min(1e-30)
        return (big * torch.sqrt(((x / big) ** 2).sum(dim=-1, keepdim=True))).squeeze(-1)


class RmsNormGamma(torch.nn.Module):
    """RMSNorm with fp32 statistics, rounded to the input dtype before the gain."""

    def forward(self, x, gamma):
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)
        return h.to(x.dtype) * gamma


class SegmentMeanPool(torch.nn.Module):
    """Embedding-bag style mean pooling over variable-length segments."""

    def forward(self, data, lengths):
        return torch.segment_reduce(data, "mean", lengths=lengths)


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def inputs_lse(device="cpu"):
    g = _gen(101)
    x = torch.randn(64, 2048, generator=g) * 2.0
    x[::16, 0] = 80.0
    return (x.to(device),)


def inputs_shifted(device="cpu"):
    return ((torch.randn(32, 3000, generator=_gen(102)) * 3.0).to(device),)


def inputs_l2(device="cpu"):
    return (torch.randn(48, 768, generator=_gen(103)).to(device),)


def inputs_rms(device="cpu"):
    g = _gen(104)
    x = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    return (x.to(device), gamma.to(device))


def inputs_segment(device="cpu"):
    g = _gen(105)
    lengths = torch.poisson(torch.full((300,), 20.0), generator=g).clamp(1, 200).to(torch.int64)
    data = torch.randn(int(lengths.sum()), 128, generator=g).to(torch.float16)
    return (data.to(device), lengths.to(device))


def inputs_wide(device="cpu"):
    return ((torch.randn(8, 65536, generator=_gen(106)) * 3.0).to(torch.bfloat16).to(device),)


# name -> (module class, input builder, apply() keyword arguments)
CASES = {
    "logsumexp_f32": (LogsumexpRows, inputs_lse, {}),
    "shifted_exp_sum_f32": (ShiftedExpSum, inputs_shifted, {}),
    "row_l2_f32": (RowL2, inputs_l2, {}),
    "rms_norm_bf16": (RmsNormGamma, inputs_rms, {"capabilities": ("rms_norm",)}),
    "segment_mean_f16": (SegmentMeanPool, inputs_segment, {"capabilities": ("segment_pool",)}),
    "logsumexp_split_bf16": (LogsumexpRows, inputs_wide, {"plan": "split"}),
}
