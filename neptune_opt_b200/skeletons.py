"""The skeleton set compiled into the CUDA library, with the scalar parameters each declares.

The reference declares its eleven scalar skeletons as sympy algebra in
neptune_codegen/library.py:19-177 and generates a Triton kernel per (skeleton, parameter values).
This backend compiles the same eleven skeletons ahead of time: each one's term, repair factor and
readout is device code (csrc/fold.cuh) and its scalar parameters are runtime arguments, so a new
value needs no compilation. This table carries what the host side needs: the C ABI id, the declared
parameters with their defaults (reference `param_defaults`, neptune_codegen/skeleton.py:255-267)
and their domains (the assumptions of the symbols in neptune_codegen/symbols.py:193-236, checked
the way algebra.py:285-302 checks them).
"""
from __future__ import annotations

import dataclasses
import math


@dataclasses.dataclass(frozen=True)
class SkeletonSpec:
    name: str
    id: int
    params: tuple = ()          # declared scalar parameters, in declaration order
    defaults: tuple = ()        # ((name, value), ...) declared defaults; others default to 1.0
    is_log: bool = False        # exponential fold with NaN/+inf status extension
    two_pass: bool = False      # no repair exists; two traversals (no split plan)
    doc: str = ""


# Parameter domains: positive symbols must be > 0, nonnegative ones >= 0, real ones finite.
DOMAINS = {"tiny": "nonnegative", "alpha": "real", "T": "positive", "beta": "positive",
           "N": "positive", "eps": "positive"}

_SPECS = (
    SkeletonSpec("logsumexp", 0, ("tiny",), (("tiny", 0.0),), True,
                 doc="softmax's max+sumexp fold, log-softmax, cross-entropy"),
    SkeletonSpec("lse_biased", 1, ("alpha", "tiny"), (("tiny", 0.0),), True,
                 doc="ALiBi-biased logsumexp: logsumexp(x + alpha)"),
    SkeletonSpec("lse_scaled", 2, ("T", "tiny"), (("T", 2.0), ("tiny", 0.0)), True,
                 doc="logsumexp(x / T): the softmax denominator for temperature-scaled logits"),
    SkeletonSpec("softcap_lse", 3, ("beta", "tiny"), (("tiny", 0.0),), True,
                 doc="soft-capped attention: logsumexp(tanh(beta*x))"),
    SkeletonSpec("stable_l2", 4, doc="numerically stable L2 norm: m * sqrt(sum((x/m)^2)), m = max|x|"),
    SkeletonSpec("linear_attn", 5, doc="linear attention normaliser: sum(x)/max|x|"),
    SkeletonSpec("decay_renorm", 6, ("N",), doc="decay renormalisation: sum(x/(N+max|x|))"),
    SkeletonSpec("sumsq_div", 7, doc="sum(x^2)/max|x|"),
    SkeletonSpec("rmsnorm_max", 8, ("eps",), doc="RMSNorm + row max: max_j x_j / sqrt(mean(x^2) + eps)"),
    SkeletonSpec("variance", 9, two_pass=True, doc="var(x, unbiased=False), two traversals"),
    SkeletonSpec("std", 10, two_pass=True, doc="std(x, unbiased=False), two traversals"),
)

SKELETONS = {s.name: s for s in _SPECS}


def supported() -> list:
    """Names of the compiled skeletons, sorted like the reference's `supported()`."""
    return sorted(SKELETONS)


def all_registered() -> list:
    return sorted(SKELETONS)


def param_defaults(name: str) -> dict:
    """Declared defaults, 1.0 for a declared parameter without one (skeleton.py:255-267)."""
    sk = SKELETONS[name]
    declared = dict(sk.defaults)
    return {p: float(declared.get(p, 1.0)) for p in sk.params}


def op_parameters(name: str) -> tuple:
    """Parameters a caller must supply (declared without a default), as the reference's
    explicit operator library requires (neptune_opt/__init__.py:557-560)."""
    sk = SKELETONS[name]
    declared = {p for p, _ in sk.defaults}
    return tuple(p for p in sk.params if p not in declared)


def checked_params(name: str, values: dict | None) -> dict:
    """Merge defaults and validate the declared parameters' domains.

    Raises KeyError for an unknown skeleton and NotImplementedError, with the reference
    certificate's wording (algebra.py:292-301), for a value outside its declared domain.
    """
    if name not in SKELETONS:
        raise KeyError(f"unknown skeleton {name!r}; have {all_registered()}")
    merged = {**param_defaults(name), **(values or {})}
    out = {}
    for p in SKELETONS[name].params:
        value = merged[p]
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise TypeError(f"parameter {p!r} must be a real number")
        value = float(value)
        if not math.isfinite(value):
            raise NotImplementedError(f"parameter {p!r} must be finite")
        if DOMAINS[p] == "positive" and value <= 0:
            raise NotImplementedError(f"parameter {p!r} must be positive")
        if DOMAINS[p] == "nonnegative" and value < 0:
            raise NotImplementedError(f"parameter {p!r} must be nonnegative")
        out[p] = value
    # Parameters the skeleton does not declare are kept (they stay part of an op's identity, as in
    # the reference) but never reach the kernel.
    for k, v in merged.items():
        out.setdefault(k, v)
    return out
