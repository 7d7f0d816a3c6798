"""The output tolerance every attention parity check uses.

The stated bar: attention output within max-abs 2e-3 (bf16/fp16) or 1e-5 (fp32)
of an fp32 reference computed from the same stored input values; LSE within
1e-3 (16-bit inputs) or 1e-5 (fp32).

A 16-bit output is the fp32 result rounded once more, to the stored type. Where
half an ulp of that type is at most 1e-3 (bf16: |O| < 0.5; fp16: |O| < 4) the
plain 2e-3 holds and is asserted as is. Above that, a stored value cannot be
within 2e-3 of every fp32 value, so the bound there is 2e-3 plus half an ulp of
the reference value (the output's own final rounding). ``band_report`` gives the
largest error per magnitude band, so the kernel's own error (the strict band)
and the rounding allowance (the bands above) are seen apart.
"""
from __future__ import annotations

import numpy as np

O_TOL = {"f32": 1e-5, "f16": 2e-3, "bf16": 2e-3}
LSE_TOL = {"f32": 1e-5, "f16": 1e-3, "bf16": 1e-3}
SIG_BITS = {"f16": 11, "bf16": 8}  # significant bits including the implicit one
BANDS = (0.0, 0.5, 1.0, 2.0, 4.0, np.inf)


def dtype_key(dtype) -> str:
    name = str(dtype)
    if "bfloat16" in name:
        return "bf16"
    if "float16" in name:
        return "f16"
    if "float32" in name:
        return "f32"
    raise ValueError(f"no tolerance for {dtype}")


def half_ulp(o_ref: np.ndarray, key: str) -> np.ndarray:
    e = np.floor(np.log2(np.maximum(np.abs(np.nan_to_num(o_ref)), 1e-30)))
    return np.exp2(e - SIG_BITS[key])


def out_tol(o_ref: np.ndarray, dtype) -> np.ndarray:
    """Per-element bound on |O - O_ref|: plain 2e-3 / 1e-5 wherever half an ulp
    of the stored type is <= 1e-3, else 2e-3 + half an ulp of O_ref."""
    key = dtype_key(dtype)
    if key == "f32":
        return np.full(np.shape(o_ref), O_TOL[key])
    h = half_ulp(o_ref, key)
    return np.where(h <= 1e-3, O_TOL[key], O_TOL[key] + h)


def strict_mask(o_ref: np.ndarray, dtype) -> np.ndarray:
    """Elements where the plain bound applies with no rounding allowance."""
    key = dtype_key(dtype)
    if key == "f32":
        return np.ones(np.shape(o_ref), dtype=bool)
    return half_ulp(o_ref, key) <= 1e-3


def band_report(o: np.ndarray, o_ref: np.ndarray) -> dict:
    """{"[lo,hi)": (count, max |O - O_ref|)} over bands of |O_ref| (NaN skipped)."""
    ok = ~np.isnan(o_ref)
    a = np.abs(o_ref[ok])
    err = np.abs(o[ok] - o_ref[ok])
    out = {}
    for lo, hi in zip(BANDS[:-1], BANDS[1:]):
        m = (a >= lo) & (a < hi)
        if m.any():
            out[f"[{lo:g},{hi:g})"] = (int(m.sum()), float(err[m].max()))
    return out


def check_out(o: np.ndarray, o_ref: np.ndarray, dtype) -> tuple[bool, str]:
    """(passes, message): NaN patterns equal and every element within out_tol."""
    nan = np.isnan(o_ref)
    if not np.array_equal(np.isnan(o), nan):
        return False, "NaN pattern differs"
    err = np.abs(np.where(nan, 0, o) - np.where(nan, 0, o_ref))
    tol = out_tol(np.where(nan, 0, o_ref), dtype)
    bad = err > tol
    if bad.any():
        return False, (f"{int(bad.sum())} of {bad.size} outputs off; worst excess {float((err - tol).max()):.3g}; "
                       f"per |O_ref| band (count, max err): {band_report(o, o_ref)}")
    return True, ""
