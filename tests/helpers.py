"""Shared comparison helpers for the parity tests."""
from __future__ import annotations

import numpy as np


def f32(bits) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def ulp_bf16(v) -> np.ndarray:
    """Spacing of bf16 at |v| (2^(e-7) for normal values)."""
    a = np.abs(np.asarray(v, dtype=np.float32))
    a = np.maximum(a, np.float32(2.0 ** -126))
    e = np.floor(np.log2(a))
    return (2.0 ** (e - 7)).astype(np.float32)


def bf16_tolerance(ref: np.ndarray, ulps: float = 2.0, rel: float = 1e-2,
                   operands=(), operand_ulps: float | None = None) -> np.ndarray:
    """Per-element tolerance of the north-star bar: the looser of `ulps` bf16
    ULP and `rel` relative, plus a floor of one bf16 ULP of max|ref|/256 for
    elements cancelled into the noise (the reference's own convention:
    engine/patches/round2/wsum10/test_exact.py counts ULPs only where
    |ref| >= max|ref|/256).

    `operands` are the bf16 terms of the output's last rounding step (the
    routed sum and the gated shared term of ``y = routed + shared``).  Where
    that add cancels, one ULP of an operand is many ULPs of the result, so
    the ULP bar is also counted on the operands: |got - ref| <= ulps * ulp(op)
    for the largest operand passes."""
    r = np.abs(ref.astype(np.float32))
    floor = ulp_bf16(np.float32(r.max() / 256.0)) if r.size else np.float32(0)
    tol = np.maximum(ulps * ulp_bf16(r), rel * r)
    ou = ulps if operand_ulps is None else operand_ulps
    for op in operands:
        tol = np.maximum(tol, ou * ulp_bf16(np.abs(f32(op))))
    return tol + floor


def assert_bf16_close(got_bits, ref_bits, ulps=2.0, rel=1e-2, what="", operands=(),
                      operand_ulps=None):
    g, r = f32(got_bits), f32(ref_bits)
    tol = bf16_tolerance(r, ulps, rel, operands, operand_ulps)
    bad = np.abs(g - r) > tol
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements outside tolerance; first at {tuple(i)}: "
            f"got {g[tuple(i)]} ref {r[tuple(i)]} tol {tol[tuple(i)]}")


def rel_rms(got, ref) -> float:
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    return float(np.sqrt(np.mean((g - r) ** 2) / (np.mean(r ** 2) + 1e-300)))
