"""Tolerances of the parity tests, restated from the reference's own tests.

* LEVEL and EXACT are kernels/gpu/tests/test_gpu_ffn.cpp:30-50: max_rel = max|got - ref| / max|ref|,
  relative L2 and cosine. LEVEL (1e-2, 1e-2, 0.9999) is for GEMV/GEMM/FFN results; EXACT
  (1e-2, 5e-3, 0.99999) for single-rounding kernels. max_rel <= 1e-2 is also the tolerance the
  build's specification sets against the CPU oracle.
* error_metrics restates experiments/ffn_partition/contract.py:172-208 (fixed limits rtol 0.03,
  atol 0.05, relative L2 0.02), used by the partition-level checks.
"""
import numpy as np

LEVEL = (1e-2, 1e-2, 0.9999)
EXACT = (1e-2, 5e-3, 0.99999)


def compare(got, ref):
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    max_rel = np.abs(g - r).max() / (np.abs(r).max() + 1e-30)
    rel_l2 = np.linalg.norm(g - r) / (np.linalg.norm(r) + 1e-30)
    cos = float(np.dot(g, r) / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-30))
    return float(max_rel), float(rel_l2), cos


def assert_close(got, ref, tol=LEVEL, what=""):
    max_rel, rel_l2, cos = compare(got, ref)
    ok = max_rel <= tol[0] and rel_l2 <= tol[1] and cos >= tol[2]
    assert ok, f"{what}: max_rel={max_rel:.2e} rel_l2={rel_l2:.2e} cos={cos:.7f} (limits {tol})"
    return max_rel, rel_l2, cos


def assert_bf16_close(got_bits, ref_bits, max_rel=2.0 ** -8, min_equal=0.99, what=""):
    """Two bf16 bit arrays from the same arithmetic in a different summation order: identical in at
    least `min_equal` of the elements, and no element further from the reference than `max_rel`
    times max|ref| (one bf16 ulp at the largest magnitude by default). A per-element ulp bound
    does not hold where a sum cancels to a small value."""
    g = np.asarray(got_bits, np.uint16).ravel()
    r = np.asarray(ref_bits, np.uint16).ravel()
    gf = (g.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    rf = (r.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    eq = float(np.mean(g == r))
    rel = float(np.abs(gf - rf).max() / (np.abs(rf).max() + 1e-30))
    assert rel <= max_rel and eq >= min_equal, f"{what}: max_rel {rel:.2e}, equal {eq:.4f}"
    return eq


def error_metrics(actual, expected, rtol=0.03, atol=0.05, l2_limit=0.02):
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    if actual.shape != expected.shape or actual.size == 0:
        raise ValueError("actual and expected must have the same nonempty shape")
    finite = bool(np.all(np.isfinite(actual)))
    if not finite:
        return {"passed": False, "finite": False}
    delta = actual.astype(np.float64) - expected.astype(np.float64)
    norm = float(np.linalg.norm(expected.astype(np.float64)))
    max_ref = float(np.max(np.abs(expected)))
    max_error = float(np.max(np.abs(delta)))
    rel_l2 = float(np.linalg.norm(delta)) / norm if norm else (0.0 if max_error == 0 else None)
    passed = (max_error == 0) if norm == 0 else (rel_l2 <= l2_limit and max_error <= atol + rtol * max_ref)
    return {"passed": bool(passed), "finite": True, "max_abs_error": max_error, "relative_l2_error": rel_l2}
