"""GPU parity of the tcgen05 attention kernel against an fp64 softmax(scale Q K^T) V.

The reference is the unfused float64 computation of the same bf16 inputs (scores, causal mask,
log-sum-exp, normalised probabilities, product with V), on whole heads for small shapes and on
sampled heads of the full [8, 32, 4096, 128] configuration.

Tolerance (bf16 output of an fp32 computation with bf16 probabilities):
  |O - O_ref| <= 2^-9 * max|V| + 2^-8 * |O_ref|
The kernel rounds each probability p to bf16 before the P V product (relative error <= 2^-9), so
the weighted mean sum(p v) / l moves by at most 2^-9 * max|v|; the final bf16 rounding of O adds at
most 2^-9 * |O| (2^-8 leaves room for the fp32 accumulation and the ex2 approximation, whose
relative errors are around 2^-22).
  |LSE - LSE_ref| <= 2e-5 * (1 + |LSE_ref|)   (fp32 scores and sums)
"""
from __future__ import annotations

import math

import pytest

from conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


def _reference(q, k, v, causal, scale):
    """fp64 O and LSE for one head: q, k, v [S, D] (any device)."""
    import torch

    s = (q.double() @ k.double().T) * scale
    if causal:
        n = s.shape[0]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    return torch.exp(s - lse[:, None]) @ v.double(), lse


def _check_head(o, lse, q, k, v, causal, scale, label):
    import torch

    ref_o, ref_lse = _reference(q, k, v, causal, scale)
    got = o.double()
    bound = 2.0 ** -9 * v.double().abs().max() + 2.0 ** -8 * ref_o.abs()
    err = (got - ref_o).abs()
    assert torch.isfinite(got).all(), f"{label}: non-finite output"
    worst = (err - bound).max().item()
    assert worst <= 0, f"{label}: |O - ref| exceeds the bound by {worst:.3g} (max err {err.max().item():.3g})"
    lerr = (lse.double() - ref_lse).abs()
    lbound = 2e-5 * (1 + ref_lse.abs())
    assert (lerr <= lbound).all(), f"{label}: LSE error {lerr.max().item():.3g}"


def _inputs(b, h, s, gen, d=128):
    import torch

    mk = lambda: torch.randn(b, h, s, d, generator=gen).to(torch.bfloat16).cuda()  # noqa: E731
    return mk(), mk(), mk()


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(1, 2, 256, 128), (2, 3, 200, 128), (1, 1, 1, 128), (1, 2, 129, 128),
                                   (1, 1, 1000, 128), (2, 1, 384, 128), (1, 1, 640, 128)])
def test_attention_matches_fp64_on_whole_heads(shape, causal):
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(hash((shape, causal)) % (2 ** 31))
    b, h, s, d = shape
    q, k, v = _inputs(b, h, s, gen, d)
    keep = (q.clone(), k.clone(), v.clone())
    scale = 1.0 / math.sqrt(d)
    o, lse = NB.attention(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    assert o.shape == q.shape and o.dtype == torch.bfloat16 and lse.shape == (b, h, s)
    for bi in range(b):
        for hi in range(h):
            _check_head(o[bi, hi], lse[bi, hi], q[bi, hi], k[bi, hi], v[bi, hi], causal, scale,
                        f"{shape} causal={causal} head ({bi},{hi})")
    for a, c in zip((q, k, v), keep):
        assert torch.equal(a, c), "inputs were modified"
    assert NB._lib.stream_fault() == 0


@pytest.mark.parametrize("direction", [1.0, -1.0])
def test_attention_online_rescale_when_the_max_moves_across_key_tiles(direction):
    """Scores that climb (or fall) by ~2^13 per 128-key tile: every tile raises the running max past
    the rescale slack (or never does), exercising the O rescale in tensor memory."""
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(7)
    s, d = 1024, 128
    q = torch.randn(1, 2, s, d, generator=gen)
    k = torch.randn(1, 2, s, d, generator=gen)
    v = torch.randn(1, 2, s, d, generator=gen)
    q[..., 0] = 6.0
    k[..., 0] = direction * torch.linspace(-6.0, 6.0, s)
    q, k, v = (t.to(torch.bfloat16).cuda() for t in (q, k, v))
    for causal in (False, True):
        o, lse = NB.attention(q, k, v, causal=causal, scale=1.0, return_lse=True)
        torch.cuda.synchronize()
        for hi in range(2):
            _check_head(o[0, hi], lse[0, hi], q[0, hi], k[0, hi], v[0, hi], causal, 1.0,
                        f"rescale dir={direction} causal={causal} head {hi}")


@pytest.mark.parametrize("causal", [False, True])
def test_attention_full_config_on_sampled_heads(causal):
    """B=8, H=32, S=4096, D=128 (the benchmark configuration): three heads checked in full, every
    output finite, and a second run bitwise identical."""
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(2024 + int(causal))
    q, k, v = _inputs(8, 32, 4096, gen)
    o, lse = NB.attention(q, k, v, causal=causal, return_lse=True)
    o2 = NB.attention(q, k, v, causal=causal)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    assert torch.equal(o, o2), "attention is not deterministic"
    scale = 1.0 / math.sqrt(128)
    for bi, hi in ((0, 0), (3, 17), (7, 31)):
        _check_head(o[bi, hi], lse[bi, hi], q[bi, hi], k[bi, hi], v[bi, hi], causal, scale,
                    f"full causal={causal} head ({bi},{hi})")
    assert NB._lib.stream_fault() == 0


def test_attention_custom_op_runs_the_kernel():
    import torch

    import neptune_opt_b200 as NB

    gen = torch.Generator().manual_seed(3)
    q, k, v = _inputs(1, 2, 300, gen)
    before = NB.launch_count()
    o, lse = NB.attention_op()(q, k, v, True, 0.1)
    torch.cuda.synchronize()
    assert NB.launch_count() == before + 1
    for hi in range(2):
        _check_head(o[0, hi], lse[0, hi], q[0, hi], k[0, hi], v[0, hi], True, 0.1, f"op head {hi}")
