"""Parity metrics shared by the tests.

The north-star tolerance is "max rel error <= 2e-3 on bf16 outputs".  A
relative error per element is ill-conditioned near zero, and one rounding
flip between two fp32-accurate results is already up to 2^-7 of an element,
so the tolerance is applied as:

* max over output vectors (rows) of ||got - ref||_2 / ||ref||_2 <= 2e-3;
* every element within 2 units in the last place of the 16-bit format of
  the reference value plus `atol_frac` times the row's RMS (an absolute floor
  for outputs near zero, whose ulp is far below the accumulation error);
* at most `max_mismatch` of the elements differ from the oracle at all.
"""
from __future__ import annotations

import numpy as np

REL_TOL = 2e-3


def half_to_f64(h: np.ndarray, dtype: int = 0) -> np.ndarray:
    h = np.asarray(h)
    h = h.view(np.uint16) if h.dtype != np.uint16 else h
    if dtype == 1:
        return h.view(np.float16).astype(np.float64)
    return (h.astype(np.uint32) << np.uint32(16)).view(np.float32).astype(np.float64)


def ulp(v: np.ndarray, dtype: int = 0) -> np.ndarray:
    mant = 10 if dtype == 1 else 7
    emin = -14 if dtype == 1 else -126
    a = np.abs(v)
    _, e = np.frexp(np.where(a > 0, a, 1.0))
    e = np.maximum(e - 1, emin)
    return np.ldexp(1.0, e - mant)


def parity_stats(got, ref, dtype: int = 0, atol_frac: float = 1e-5) -> dict:
    g = half_to_f64(got, dtype)
    r = half_to_f64(ref, dtype)
    g2 = g.reshape(-1, g.shape[-1]) if g.ndim > 1 else g.reshape(1, -1)
    r2 = r.reshape(g2.shape)
    num = np.sqrt(((g2 - r2) ** 2).sum(axis=1))
    den = np.sqrt((r2 ** 2).sum(axis=1))
    rel = np.where(den > 0, num / np.maximum(den, 1e-300), num)
    rms = np.sqrt((r2 ** 2).mean(axis=1, keepdims=True))
    err = np.abs(g2 - r2)
    bound = 2 * ulp(r2, dtype) + atol_frac * rms + 1e-30
    gb = np.asarray(got).view(np.uint16).reshape(g2.shape)
    rb = np.asarray(ref).view(np.uint16).reshape(g2.shape)
    return {
        "max_rel_l2": float(rel.max()) if rel.size else 0.0,
        "max_abs": float(err.max()) if err.size else 0.0,
        "ulp_violations": int((err > bound).sum()),
        "mismatch_frac": float((gb != rb).mean()) if err.size else 0.0,
    }


def assert_ffn_parity(got, ref, down_ref, scores, dtype: int = 0, what: str = "",
                      rel_tol: float = REL_TOL, max_mismatch: float = 0.05) -> dict:
    """End-to-end FFN output check.  Each staged rounding of the reference
    path (up||gate, SwiGLU, down) may legitimately land one ulp apart when the
    two implementations' fp32-accurate values straddle a rounding boundary;
    a flip of down[m,k,h] moves y[m,h] by score[m,k] * ulp(down[m,k,h]).  The
    per-element bound is therefore 2 ulp(y) + 2 * sum_k score_k * ulp(down_k)
    (+ 1e-5 of the row RMS); rel-L2 per row stays <= 2e-3."""
    g = half_to_f64(got, dtype)
    r = half_to_f64(ref, dtype)
    M, H = r.shape
    d = half_to_f64(down_ref, dtype).reshape(M, -1, H)
    sc = np.asarray(scores, np.float64).reshape(M, -1, 1)
    prop = 2.0 * (sc * ulp(d, dtype)).sum(axis=1)
    rms = np.sqrt((r ** 2).mean(axis=1, keepdims=True))
    bound = 2 * ulp(r, dtype) + prop + 1e-5 * rms
    err = np.abs(g - r)
    rel = np.sqrt(((g - r) ** 2).sum(axis=1)) / np.maximum(np.sqrt((r ** 2).sum(axis=1)), 1e-300)
    st = {"max_rel_l2": float(rel.max()), "max_abs": float(err.max()),
          "bound_violations": int((err > bound).sum()),
          "mismatch_frac": float((np.asarray(got).view(np.uint16) !=
                                  np.asarray(ref).view(np.uint16)).mean())}
    assert st["max_rel_l2"] <= rel_tol, f"{what}: {st}"
    assert st["bound_violations"] == 0, f"{what}: {st}"
    assert st["mismatch_frac"] <= max_mismatch, f"{what}: {st}"
    return st


def assert_parity(got, ref, dtype: int = 0, what: str = "", rel_tol: float = REL_TOL,
                  max_mismatch: float = 0.02, atol_frac: float = 1e-5) -> dict:
    st = parity_stats(got, ref, dtype, atol_frac)
    assert st["max_rel_l2"] <= rel_tol, f"{what}: {st}"
    assert st["ulp_violations"] == 0, f"{what}: {st}"
    assert st["mismatch_frac"] <= max_mismatch, f"{what}: {st}"
    return st
