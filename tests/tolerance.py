"""The parity bar of the GPU tests, in one place.

bf16 results: relative-L2 <= 5e-3 and, element by element,

    |got - ref| <= 2e-2 + u(ref)

where u(ref) is half a unit in the last place of a bf16 number of ref's magnitude,
2^(floor(log2 |ref|) - 8): the error of rounding the exact result to the bf16 output
dtype, which no kernel with a bf16 output can avoid (it alone exceeds 2e-2 once
|ref| >= 8).  This is the north-star bar (max-abs <= 2e-2, rel-L2 <= 5e-3) plus exactly
the output's own rounding, and nothing else: no quantile, no per-tensor relaxation.

fp32 results: |got - ref| <= 2e-4 and relative-L2 <= 1e-5 (no rounding term).
"""
from __future__ import annotations

import math

import numpy as np

BF16_ATOL, BF16_REL_L2 = 2e-2, 5e-3
F32_ATOL, F32_REL_L2 = 2e-4, 1e-5


def bf16_half_ulp(ref: np.ndarray) -> np.ndarray:
    """Half an ulp of bf16 at |ref| (0 where ref == 0)."""
    a = np.abs(np.asarray(ref, dtype=np.float64))
    _, e = np.frexp(a)  # a = m * 2^e, m in [0.5, 1): floor(log2 a) = e - 1
    return np.where(a > 0, np.ldexp(1.0, e - 9), 0.0)


def stats(got, ref, bf16: bool = True) -> dict:
    """max-abs, worst excess over the per-element bound, rel-L2 and the pass verdict."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    atol, rtol = (BF16_ATOL, BF16_REL_L2) if bf16 else (F32_ATOL, F32_REL_L2)
    diff = np.abs(got - ref)
    if not diff.size:
        return {"max_abs": 0.0, "excess": -atol, "rel_l2": 0.0, "pass": True}
    bound = atol + (bf16_half_ulp(ref) if bf16 else 0.0)
    # rel-L2 with a floor of atol*sqrt(n) on ||ref||, so an all-(near-)zero reference
    # (e.g. dq of a length-1 sequence) is judged by the absolute bound alone
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), atol * math.sqrt(ref.size)))
    excess = float((diff - bound).max())
    return {"max_abs": float(diff.max()), "excess": excess, "rel_l2": rel, "pass": excess <= 0 and rel <= rtol}


def assert_close(name: str, got, ref, bf16: bool = True) -> None:
    s = stats(got, ref, bf16)
    rule = "2e-2 + half-ulp(bf16)" if bf16 else "2e-4"
    assert s["pass"], (f"{name}: max-abs {s['max_abs']:.3e} (bound {rule}, worst excess {s['excess']:.2e}), "
                       f"rel-L2 {s['rel_l2']:.3e} (<= {BF16_REL_L2 if bf16 else F32_REL_L2})")
