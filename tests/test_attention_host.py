"""Host-side contract of the attention entry point (no GPU): exception types before any launch,
shape-only fake kernel of the registered op."""
from __future__ import annotations

import pytest


def _meta(*shape, dtype=None):
    import torch

    return torch.empty(*shape, dtype=dtype or torch.bfloat16, device="meta")


def test_attention_validation_raises_the_backend_exception_types():
    import torch

    import neptune_opt_b200 as NB

    q = _meta(2, 3, 256, 128)
    with pytest.raises(TypeError):
        NB.attention(q.to(torch.float16), q.to(torch.float16), q.to(torch.float16))
    with pytest.raises(ValueError):
        NB.attention(q, q, _meta(2, 3, 128, 128))
    with pytest.raises(ValueError):
        NB.attention(q[0], q[0], q[0])
    with pytest.raises(NotImplementedError):
        NB.attention(_meta(1, 1, 64, 64), _meta(1, 1, 64, 64), _meta(1, 1, 64, 64))
    with pytest.raises(ValueError):
        NB.attention(q, q, q, scale=0.0)
    cpu = torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        NB.attention(cpu, cpu, cpu)


def test_attention_op_fake_kernel_gives_shapes_only():
    import torch

    import neptune_opt_b200 as NB

    op = NB.attention_op()
    assert isinstance(op, torch._ops.OpOverload)
    q = _meta(2, 4, 300, 128)
    o, lse = op(q, q, q, True, 0.125)
    assert o.shape == q.shape and o.dtype == torch.bfloat16
    assert lse.shape == (2, 4, 300) and lse.dtype == torch.float32
