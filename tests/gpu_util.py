"""Shared helpers for the GPU parity tests (import only from -m gpu tests)."""
import numpy as np


def gemm_ref(a, b):
    """float64 product and the elementwise scale |A| @ |B| for error bounds."""
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    return a64 @ b64, np.abs(a64) @ np.abs(b64)


def assert_fp32_gemm(c, a, b, tol=1e-5):
    """FP32-accurate: every element within tol * (|A||B|)_ij of the exact
    product.  FP32 accumulation of up to 16384 terms (on the CPU or inside the
    tensor core's fp32 accumulator) sits inside this; a TF32-only product,
    whose per-product error is ~2^-11, misses it by ~50x."""
    exact, scale = gemm_ref(a, b)
    err = np.abs(c.astype(np.float64) - exact)
    bound = tol * scale + 1e-30
    worst = float(np.max(err / bound))
    assert worst <= 1.0, f"max error {worst:.3g} x bound (tol {tol})"


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
