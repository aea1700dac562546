"""CPU ORACLE -- test infrastructure only: the reference's unfused ATen graphs, run on the host.

What the reference (Defyli/neptune-opt) executes when no fused region is used -- its fallback
and the baseline its A/B gate compiles -- is the user's graph of ATen operators. On the host these
are torch's own CPU kernels. This module restates those graphs op for op (no fusion, the same
dtype conversions), so that bench.py's reference arm times the reference's CPU path itself on the
full benchmark configuration, with all host threads torch is allowed to use.

Pinned by tests/test_oracle_golden.py against vectors the reference produced
(tests/golden/make_golden.py): rms_norm is bit-identical to the reference's RMSNorm outputs.
Only tests/ and bench.py's CPU legs use this module; the product path never imports it.
"""
from __future__ import annotations


def rms_norm(x, gamma, eps: float = 1e-6):
    """The ATen RMSNorm graph of the reference's structured tests (tests/test_recognize.py:595-597;
    the same stages as emitters.py:576-595): fp32 statistics, a rounding to the input dtype, then
    the gain in the input dtype."""
    import torch

    z = x.float()
    return (z * torch.rsqrt(z.square().mean(-1, keepdim=True) + eps)).to(x.dtype) * gamma.to(x.dtype)


def logsumexp(x, dim: int = -1):
    """The lowering of logsumexp into the reference's two dependent reductions
    (neptune_recognize/lowering.py:80-90): fp32 accumulation, max with +-inf guarded to zero,
    sum of exponentials of the centred values, log, add back."""
    import torch

    t = x.float() if x.dtype in (torch.float16, torch.bfloat16) else x
    m = t.amax(dim, keepdim=True)
    m_safe = torch.where(m.abs() == float("inf"), 0.0, m)
    lse = m_safe + torch.log(torch.exp(t - m_safe).sum(dim, keepdim=True))
    return lse.squeeze(dim).to(x.dtype)


def segment_pool(data, lengths, reduce: str):
    """torch.segment_reduce over lengths: the ATen operator the reference's structured segment
    regions replace (neptune_codegen/torch_op.py:286-306 reproduces its rounding order)."""
    import torch

    return torch.segment_reduce(data, reduce, lengths=lengths)
