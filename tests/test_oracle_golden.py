"""The CPU oracle against vectors the reference itself produced (tests/golden/make_golden.py).

This pins the oracle before it is trusted as the GPU kernels' checker: every serial-fold, split-plan,
two-pass, softmax, RMSNorm, segment-pooling and span case recorded from the reference must be
reproduced -- bit-exactly for segment pooling and spans, within fp32 summation-order tolerance for
the floating-point folds.
"""
from __future__ import annotations

import ast

import numpy as np
import pytest

from conftest import assert_close_dtype, assert_nonfinite_equal, assert_rms_close, golden, round_to

pytestmark = pytest.mark.filterwarnings("ignore::RuntimeWarning")


def _fold_cases():
    data = golden("fold.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in data.files})
    return data, keys


def test_fold_serial_and_split_match_reference_kernels(oracle_mod):
    data, keys = _fold_cases()
    assert len(keys) >= 75
    for key in keys:
        name, _pi, label, dtype = key.split("|")
        x = data[key + "|x"]
        params = dict(ast.literal_eval(str(data[key + "|params"])))
        got = oracle_mod.fold(name, x, params, block=256)
        # fp32 results of the reference's own kernel (before narrowing): summation order differs
        # (tree within a chunk there, sequential here), so 1e-5 relative plus a cancellation floor.
        ref = data[key + "|serial"]
        scale = np.nanmax(np.abs(np.where(np.isfinite(ref), ref, 0))) if ref.size else 0
        assert_close_dtype(got, ref, "float32", rtol32=1e-5, atol32=1e-6 * (1 + scale))
        # and after narrowing to the input dtype they agree to 1 ulp
        assert_close_dtype(round_to(got, dtype), round_to(ref, dtype), dtype if dtype != "float32" else "float32",
                           rtol32=1e-5, atol32=1e-6 * (1 + scale))
        if key + "|split" in data.files:
            block = int(data[key + "|split_block"])
            states = oracle_mod.partial(name, x, params, 0, x.shape[1], block)
            got2 = oracle_mod.merge(name, states, params)
            assert_close_dtype(got2, data[key + "|split"], "float32", rtol32=1e-5, atol32=1e-6 * (1 + scale))


def test_fold_matches_reference_aten_oracles(oracle_mod):
    data, keys = _fold_cases()
    for key in keys:
        if key + "|graph_reference" not in data.files:
            continue
        name = key.split("|")[0]
        x = data[key + "|x"]
        params = dict(ast.literal_eval(str(data[key + "|params"])))
        got = oracle_mod.fold(name, x, params, block=1024)
        for which in ("graph_reference", "reference"):
            ref = data[key + "|" + which]
            scale = float(np.max(np.abs(ref)))
            assert_close_dtype(got, ref, "float32", rtol32=2e-5, atol32=2e-6 * (1 + scale))


def test_log_family_nonfinite_status_rows_exact(oracle_mod):
    """NaN beats +inf, +inf beats finite, all -inf gives -inf (emitters.py:522-532)."""
    data, keys = _fold_cases()
    n = 0
    for key in keys:
        if "|special|" not in key:
            continue
        name = key.split("|")[0]
        params = dict(ast.literal_eval(str(data[key + "|params"])))
        got = oracle_mod.fold(name, data[key + "|x"], params, block=256)
        assert_nonfinite_equal(got, data[key + "|serial"])
        n += 1
    assert n >= 24


def test_softmax_family_matches_torch_semantics(oracle_mod):
    sm = golden("softmax.npz")
    x = sm["x"]
    y, lse = oracle_mod.softmax(x, log=False)
    assert_close_dtype(y, sm["softmax"], "float32", rtol32=1e-5, atol32=1e-30)
    ly, _ = oracle_mod.softmax(x, log=True)
    assert_close_dtype(ly, sm["log_softmax"], "float32", rtol32=1e-5, atol32=1e-5)
    assert_close_dtype(lse, sm["logsumexp"], "float32", rtol32=1e-5, atol32=1e-6)


def test_rms_norm_matches_reference_aten_form(oracle_mod):
    rms = golden("rms_norm.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in rms.files})
    for key in keys:
        dtype = key.split("|")[0]
        got = oracle_mod.rms_norm(rms[key + "|x"], rms[key + "|gamma"], 1e-6, dtype)
        assert_rms_close(got, rms[key + "|out"], dtype)


def test_aten_graph_restatements_match_the_reference_outputs():
    """oracle/aten_graph.py (the reference arm's CPU path): bit-identical to the reference's RMSNorm
    ATen outputs and segment outputs, and its logsumexp lowering within fp32 rounding of the
    reference's ATen logsumexp."""
    import torch

    from oracle import aten_graph

    rms = golden("rms_norm.npz")
    for key in sorted({k.rsplit("|", 1)[0] for k in rms.files}):
        dt = getattr(torch, key.split("|")[0])
        x = torch.from_numpy(rms[key + "|x"]).to(dt)
        g = torch.from_numpy(rms[key + "|gamma"]).to(dt)
        got = aten_graph.rms_norm(x, g, 1e-6).float().numpy()
        assert np.array_equal(got, rms[key + "|out"]), key
    sm = golden("softmax.npz")
    x = torch.from_numpy(sm["x"])
    fin = np.isfinite(sm["logsumexp"])
    got = aten_graph.logsumexp(x).numpy()
    assert np.array_equal(np.isnan(got), np.isnan(sm["logsumexp"]))
    np.testing.assert_allclose(got[fin], sm["logsumexp"][fin], rtol=1e-6)
    seg = golden("segment.npz")
    for key in sorted({k.rsplit("|", 1)[0] for k in seg.files}):
        dtype, view, initial, reduce, kind = key.split("|")
        if kind != "len" or initial != "None" or view != "poisson":
            continue
        data = torch.from_numpy(seg[key + "|data"]).to(getattr(torch, dtype))
        lengths = torch.from_numpy(seg[key + "|segments"])
        got = aten_graph.segment_pool(data, lengths, reduce).float().numpy()
        ref = seg[key + "|out"]
        assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(got[~np.isnan(ref)],
                                                                              ref[~np.isnan(ref)]), key


def test_segment_pool_bit_exact_against_reference(oracle_mod):
    seg = golden("segment.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in seg.files})
    assert len(keys) >= 80
    for key in keys:
        dtype, _view, initial, reduce, kind = key.split("|")
        initial = None if initial == "None" else float(initial)
        data = seg[key + "|data"]
        spans, status = oracle_mod.segment_spans(seg[key + "|segments"], kind == "off", False, data.shape[0])
        assert status == 0
        got = oracle_mod.segment_pool(data, spans, reduce, initial, dtype)
        ref = seg[key + "|out"]
        np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
        np.testing.assert_array_equal(got[~np.isnan(ref)], ref[~np.isnan(ref)])
        fin = ~np.isnan(ref)
        np.testing.assert_array_equal(np.signbit(got[fin]), np.signbit(ref[fin]))  # -0.0 stays -0.0
        if key + "|reference_kernel" in seg.files:
            np.testing.assert_array_equal(got, seg[key + "|reference_kernel"])


def test_segment_spans_match_reference_assertions(oracle_mod):
    from neptune_opt_b200.torch_op import SPAN_MESSAGES

    sp = golden("spans.npz")
    labels = sorted({k.rsplit("|", 1)[0] for k in sp.files})
    for label in labels:
        is_off, unsafe, nrows = (int(v) for v in sp[label + "|meta"])
        segs = sp[label + "|segments"]
        spans, status = oracle_mod.segment_spans(segs, bool(is_off), bool(unsafe), nrows)
        error = str(sp[label + "|error"])
        if not error:
            assert status == 0, label
            np.testing.assert_array_equal(spans, sp[label + "|spans"])
        else:
            first = next(msg for bit, msg in SPAN_MESSAGES if status & bit)
            assert first in error, (label, first, error)


def test_round_dtype_matches_torch_rtne(oracle_mod):
    rng = np.random.default_rng(0)
    x = np.concatenate([(rng.standard_normal(20000) * 10.0 ** rng.integers(-8, 6, 20000)).astype(np.float32),
                        np.array([65504, 65519.99, 65520, 1e-40, -0.0, 6e-8, 3e38, -3.4e38], np.float32)])
    for dtype in ("bfloat16", "float16"):
        np.testing.assert_array_equal(oracle_mod.round_dtype(x, dtype), round_to(x, dtype))


@pytest.mark.parametrize("causal", [False, True])
def test_attention_oracle_agrees_with_torch_sdpa_on_cpu(causal):
    """The fp64 attention checker against torch's own CPU scaled_dot_product_attention (math
    backend, float64) on bf16-valued inputs, including a ragged length."""
    import torch

    import oracle

    gen = torch.Generator().manual_seed(11)
    for s in (1, 37, 130):
        q, k, v = (torch.randn(2, 3, s, 128, generator=gen).to(torch.bfloat16).double() for _ in range(3))
        want = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal).numpy()
        got, lse = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=causal)
        np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
        assert lse.shape == (2, 3, s) and np.all(np.isfinite(lse))
