"""Parity criteria (stated once, used by every parity test).

- Elementwise / view / indexing graphs: bit-exact (NaNs compared as a class).
- Reductions, softmax, exp-based graphs: relative error <= 1e-5 per element,
  i.e. |got - want| <= 1e-5 * max(|want|, 1e-30) + 1e-30.
- Sums over many terms that can cancel (a reduction of signed values):
  |got - want| <= 1e-5 * max(|want|, sum|x| / sqrt(n)) per output, i.e.
  relative to the sum's own scale (sqrt(n) times the typical term), since a
  sum that cancels to near zero has no fp32 evaluation order that meets a
  bound relative to its tiny result.
- fp32 matmul: per element |C - C64| / (max(|C64|, rms(C64)) * sqrt(K)) <= 1e-5
  against an fp64 reference C64 (the 1e-5 "relative, normalised by sqrt(K)"
  criterion); plus a sharper check in the matmul tests that the error stays
  within a small multiple of an fp32 FMA chain's own error, so a plain
  single-pass TF32 product would fail.
"""

import numpy as np

REL_TOL = 1e-5
MATMUL_TOL = 1e-5


def assert_bitwise(got: np.ndarray, want: np.ndarray, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float32).reshape(-1)
    want = np.asarray(want, dtype=np.float32).reshape(-1)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    gb = got.view(np.uint32)
    wb = want.view(np.uint32)
    both_nan = np.isnan(got) & np.isnan(want)
    bad = (gb != wb) & ~both_nan
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} of {got.size} differ; first at {i}: "
                             f"got {got[i]!r} ({gb[i]:08x}) want {want[i]!r} ({wb[i]:08x})")


def assert_relative(got: np.ndarray, want: np.ndarray, tol: float = REL_TOL, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    both_nan = np.isnan(got) & np.isnan(want)
    same_inf = np.isinf(got) & np.isinf(want) & (np.sign(got) == np.sign(want))
    err = np.abs(got - want)
    bound = tol * np.maximum(np.abs(want), 1e-30) + 1e-30
    bad = ~(both_nan | same_inf | (err <= bound))
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} of {got.size} exceed rel {tol}; first at {i}: "
                             f"got {got[i]!r} want {want[i]!r} rel {err[i] / max(abs(want[i]), 1e-30):.3e}")


def assert_sum_close(got: np.ndarray, want: np.ndarray, abs_sum: np.ndarray, n: int,
                     tol: float = REL_TOL, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    scale = np.maximum(np.abs(want), np.asarray(abs_sum, dtype=np.float64).reshape(-1) / np.sqrt(max(n, 1)))
    err = np.abs(got - want)
    bad = err > tol * scale + 1e-30
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} of {got.size} exceed {tol} of the sum's scale; "
                             f"first at {i}: got {got[i]!r} want {want[i]!r} scale {scale[i]:.4g}")


def matmul_error(got: np.ndarray, want64: np.ndarray, k: int) -> float:
    got = np.asarray(got, dtype=np.float64)
    want64 = np.asarray(want64, dtype=np.float64)
    rms = float(np.sqrt(np.mean(want64 * want64))) if want64.size else 0.0
    scale = np.maximum(np.abs(want64), rms) * np.sqrt(k)
    scale = np.where(scale == 0, 1.0, scale)
    return float(np.max(np.abs(got - want64) / scale)) if got.size else 0.0
