"""Generate the golden vectors in tests/golden/ from the reference implementation itself.

Run where a checkout of the reference (Defyli/neptune-opt) is importable, e.g.

    python tests/golden/make_golden.py /path/to/neptune-opt

The reference's own generated Triton kernels are executed on the CPU with Triton's interpreter
(TRITON_INTERPRET=1): the serial fold (neptune_codegen/template.py:41-54), the split pair
(template.py:137-165), the two-pass plan (template.py:62-103) and the ordered segment kernel
(neptune_codegen/torch_op.py:286-306). Their fp32 results are recorded before any narrowing
(the interpreter's own bf16 store is not round-to-nearest-even, so kernels write into fp32
buffers and the tests narrow with torch's RTNE conversion). Alongside them the script records the
reference's ATen oracles (neptune_codegen/references.py:57-140), the RMSNorm ATen form of
tests/test_recognize.py:595-597, torch.segment_reduce on the reference's segment test cases
(tests/test_autotune.py:794-833) and the outcome of the reference's span assertions
(torch_op.py:370-387) on valid and invalid descriptors.

Inputs are small and seeded, so the fixtures stay a few hundred KB.
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}

# Non-default parameter values exercised besides each skeleton's declared defaults.
EXTRA_PARAMS = {
    "logsumexp": {"tiny": 1e-6},
    "lse_biased": {"alpha": -0.75, "tiny": 0.0},
    "lse_scaled": {"T": 3.0, "tiny": 0.0},
    "softcap_lse": {"beta": 0.3, "tiny": 0.0},
    "decay_renorm": {"N": 2.5},
    "rmsnorm_max": {"eps": 1e-6},
}


def log_special_rows(width: int = 7) -> np.ndarray:
    nan, inf = float("nan"), float("inf")
    rows = [
        [nan, inf, 1.0],
        [inf, -inf, 1.0],
        [-inf, -inf, -inf],
        [0.0, -100.0, -200.0],
        [-inf, 1.0, 2.0],
        [80.0, 0.5, -0.5],
        [inf, 2.0, 3.0],
        [-120.0, -121.0, -119.5],
    ]
    out = np.full((len(rows), width), -inf, np.float32)
    for i, r in enumerate(rows):
        out[i, :len(r)] = r
        if i in (3, 5, 7):  # finite rows: fill the rest with finite values
            out[i, len(r):] = np.linspace(-3, 3, width - len(r))
    return out


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    import neptune_codegen as CG
    import neptune_codegen.torch_op as TO

    g = torch.Generator().manual_seed(1234)
    fold = {}
    names = CG.supported()
    base = (torch.randn(5, 1000, generator=g) * 2.0).float()
    base[1, 17] = 9.0
    base[3] = base[3].abs() + 0.25
    special = torch.from_numpy(log_special_rows())
    cases = 0
    for name in names:
        sk = CG.SKELETONS[name]
        param_sets = [CG.param_defaults(name)]
        if name in EXTRA_PARAMS:
            param_sets.append({**CG.param_defaults(name), **EXTRA_PARAMS[name]})
        for pi, params in enumerate(param_sets):
            inputs = [("rand", base)]
            if sk.is_log:
                inputs.append(("special", special))
            for label, x32 in inputs:
                for dname, dt in DTYPES.items():
                    x = x32.to(dt)
                    rows, ncols = x.shape
                    key = f"{name}|{pi}|{label}|{dname}"
                    serial = CG.compile_skeleton(name, params)
                    out = torch.empty(rows, dtype=torch.float32)
                    serial[(rows,)](x, out, rows, ncols, x.stride(0), x.stride(1), BLOCK=256)
                    fold[key + "|x"] = x.float().numpy()
                    fold[key + "|serial"] = out.numpy().copy()
                    if not sk.two_pass:
                        partial, merge = CG.compile_skeleton(name, params, plan="split")
                        block = 128 if ncols > 128 else 2
                        nparts, mb = CG.split_launch_shape(ncols, block)
                        pm = torch.empty(rows, nparts)
                        pa = torch.empty(rows, nparts)
                        pv = torch.empty(rows, nparts, dtype=torch.int32)
                        ps = torch.empty(rows, nparts, dtype=torch.int32)
                        partial[(rows, nparts)](x, pm, pa, pv, ps, rows, ncols, x.stride(0), x.stride(1),
                                                nparts, BLOCK=block)
                        out2 = torch.empty(rows, dtype=torch.float32)
                        merge[(rows,)](pm, pa, pv, ps, out2, rows, ncols, nparts, MERGE_BLOCK=mb)
                        fold[key + "|split"] = out2.numpy().copy()
                        fold[key + "|split_block"] = np.array(block)
                    if label == "rand":
                        fold[key + "|graph_reference"] = CG.graph_reference(name, x.float(), **params).numpy()
                        fold[key + "|reference"] = CG.reference(name, x.float(), **params).numpy()
                    fold[key + "|params"] = np.array(repr(sorted(params.items())))
                    cases += 1
    np.savez_compressed(os.path.join(HERE, "fold.npz"), **fold)
    print(f"fold: {cases} cases")

    # softmax family: the semantics the reference's lowering reproduces (lowering.py:80-99)
    sm = {}
    xs = torch.cat([base[:, :257], torch.from_numpy(np.pad(log_special_rows(), ((0, 0), (0, 250)),
                                                          constant_values=-np.inf))], 0)
    sm["x"] = xs.numpy()
    sm["softmax"] = torch.softmax(xs, -1).numpy()
    sm["log_softmax"] = torch.log_softmax(xs, -1).numpy()
    sm["logsumexp"] = torch.logsumexp(xs, -1).numpy()
    np.savez_compressed(os.path.join(HERE, "softmax.npz"), **sm)

    # RMSNorm: the ATen form the reference's structured tests check against.
    rms = {}
    for dname, dt in DTYPES.items():
        for shape in ((7, 300), (3, 4096)):
            x = (torch.randn(*shape, generator=g)).to(dt)
            gamma = (1.0 + 0.1 * torch.randn(shape[1], generator=g)).to(dt)
            eps = 1e-6
            z = x.float()
            ref = (z * torch.rsqrt((z * z).mean(-1, keepdim=True) + eps)).to(dt) * gamma
            key = f"{dname}|{shape[0]}x{shape[1]}"
            rms[key + "|x"] = x.float().numpy()
            rms[key + "|gamma"] = gamma.float().numpy()
            rms[key + "|out"] = ref.float().numpy()
    np.savez_compressed(os.path.join(HERE, "rms_norm.npz"), **rms)

    # Segments: the reference's own CUDA-test cases, run with torch.segment_reduce on CPU and, for
    # the storage types the interpreter rounds faithfully, with the reference's generated kernel.
    seg = {}
    n_seg_cases = 0
    for dname, dt in DTYPES.items():
        data0 = torch.full((1027, 2, 6), 0.1, dtype=dt)
        data0[1, 0, 0] = float("inf")
        data0[2, 0, 0] = -float("inf")
        data0[3, 1, 2] = float("nan")
        data0[4, 1, 4] = -float("inf")
        lengths = torch.tensor([0, 999, 2, 999, 1025, 999, 0, 999], dtype=torch.int32)[::2]
        offsets = torch.tensor([1, 999, 1, 999, 3, 999, 1026, 999], dtype=torch.int64)[::2]
        rnd = torch.randn(300, 5, generator=g).to(dt)
        lens_rnd = torch.poisson(torch.full((40,), 6.0), generator=g).clamp(1, 20).to(torch.int64)
        lens_rnd[-1] += 300 - int(lens_rnd.sum()) if int(lens_rnd.sum()) < 300 else 0
        for view_name, data in (("strided", data0[:, :, ::2]), ("transposed", data0.transpose(1, 2))):
            for initial in (None, 0.0, -2.125):
                for reduce in ("sum", "mean"):
                    for segs, is_off in ((lengths, False), (offsets, True)):
                        kw = {("offsets" if is_off else "lengths"): segs}
                        exp = torch.segment_reduce(data, reduce, initial=initial, **kw)
                        key = f"{dname}|{view_name}|{initial}|{reduce}|{'off' if is_off else 'len'}"
                        seg[key + "|data"] = data.float().numpy()
                        seg[key + "|segments"] = segs.numpy().astype(np.int64)
                        seg[key + "|out"] = exp.float().numpy()
                        n_seg_cases += 1
        # signed zero and subnormal (test_autotune.py:822-829)
        tiny = torch.tensor([[1e-40, -0.0], [1e-40, 0.0]], dtype=dt)
        for reduce in ("sum", "mean"):
            exp = torch.segment_reduce(tiny, reduce, lengths=torch.tensor([0, 2]), initial=-0.0)
            key = f"{dname}|signed_zero|-0.0|{reduce}|len"
            seg[key + "|data"] = tiny.float().numpy()
            seg[key + "|segments"] = np.array([0, 2], np.int64)
            seg[key + "|out"] = exp.float().numpy()
            n_seg_cases += 1
        # random segment lengths, compared against the reference's generated kernel too
        if int(lens_rnd.sum()) == 300:
            for reduce in ("sum", "mean"):
                exp = torch.segment_reduce(rnd, reduce, lengths=lens_rnd)
                key = f"{dname}|poisson|None|{reduce}|len"
                seg[key + "|data"] = rnd.float().numpy()
                seg[key + "|segments"] = lens_rnd.numpy()
                seg[key + "|out"] = exp.float().numpy()
                if dt != torch.bfloat16:
                    kernel = TO.compile_segment_reduction("segment_" + reduce,
                                                          {"initial": None, "offsets": False, "unsafe": False})
                    spans = torch.cat([torch.zeros(1, dtype=torch.int64), lens_rnd.cumsum(0)])
                    out = torch.empty(len(lens_rnd), 5, dtype=dt)
                    kernel[(len(lens_rnd), 1)](rnd, spans, out, 300, 5, len(lens_rnd), rnd.stride(0),
                                               rnd.stride(1), spans.stride(0), BLOCK=64)
                    seg[key + "|reference_kernel"] = out.float().numpy()
                n_seg_cases += 1
    np.savez_compressed(os.path.join(HERE, "segment.npz"), **seg)
    print(f"segment: {n_seg_cases} cases")

    # Span construction: cumsum for valid descriptors, first failing assertion for invalid ones.
    spans = {}
    span_cases = [
        ("len_ok", [3, 0, 4], False, False, 7),
        ("len_neg", [3, -1, 5], False, False, 7),
        ("len_big", [3, 9], False, False, 7),
        ("len_short", [3, 2], False, False, 7),
        ("len_short_unsafe", [3, 2], False, True, 7),
        ("off_ok", [0, 2, 2, 7], True, False, 7),
        ("off_oob", [0, 2, 9], True, False, 7),
        ("off_neg", [-1, 2, 7], True, False, 7),
        ("off_nonmono", [0, 5, 3, 7], True, False, 7),
        ("len_empty_rows0", [], False, False, 0),
    ]
    for label, segs, is_off, unsafe, nrows in span_cases:
        data = torch.zeros(nrows, 2)
        s = torch.tensor(segs, dtype=torch.int64)
        try:
            out = TO._segment_spans(data, s, offsets=is_off, unsafe=unsafe)
            spans[label + "|spans"] = out.numpy()
            spans[label + "|error"] = np.array("")
        except RuntimeError as exc:
            spans[label + "|spans"] = np.zeros(0, np.int64)
            spans[label + "|error"] = np.array(str(exc).splitlines()[0])
        spans[label + "|segments"] = s.numpy()
        spans[label + "|meta"] = np.array([int(is_off), int(unsafe), nrows])
    np.savez_compressed(os.path.join(HERE, "spans.npz"), **spans)
    print(f"spans: {len(span_cases)} cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NEPTUNE_REFERENCE", "."))
