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


def f64_forward_backward(dims, params, x, t, masks=None):
    """The step's exact values: forward, softmax cross-entropy (mean over the
    batch) and backward of Sequential(Linear, ReLU, ..., Linear) in float64,
    from the same float32 inputs and parameters.  Gradients come back in
    Module.parameters() order (W0, b0, W1, b1, ...), with the ReLU masks taken
    from the pre-activation as the reference's ReluBackward does
    (orca-autograd/src/backend.rs:1624-1646).

    masks (optional): one boolean array per hidden layer, the ReLU pattern to
    use instead of the float64 sign of each pre-activation -- the pattern an
    FP32 step actually used.  A pre-activation within rounding distance of
    zero can take either sign under any correct FP32 summation order (the
    reference's included); with the FP32 step's own pattern the remaining
    difference is the arithmetic alone.

    Returns (loss, grads, logits, pre) with pre the float64 pre-activations
    of the hidden layers."""
    L = len(dims) - 1
    acts = [np.asarray(x, np.float64)]
    pre, used = [], []
    Ws = [np.asarray(params[2 * l], np.float64) for l in range(L)]
    for l in range(L):
        z = acts[-1] @ Ws[l] + np.asarray(params[2 * l + 1], np.float64)
        if l + 1 < L:
            pre.append(z)
            mask = (z > 0.0) if masks is None else np.asarray(masks[l], bool)
            used.append(mask)
            acts.append(np.where(mask, z, 0.0))
        else:
            P = z
    T = np.asarray(t, np.float64)
    B = P.shape[0]
    m = P.max(axis=1, keepdims=True)
    e = np.exp(P - m)
    s = e.sum(axis=1, keepdims=True)
    loss = float(-(T * (P - m - np.log(s))).sum() / B)
    g = (e / s * T.sum(axis=1, keepdims=True) - T) / B
    grads = [None] * (2 * L)
    for l in range(L - 1, -1, -1):
        grads[2 * l] = acts[l].T @ g
        grads[2 * l + 1] = g.sum(axis=0, keepdims=True)
        if l > 0:
            g = (g @ Ws[l].T) * used[l - 1]
    return loss, grads, P, pre


def gpu_masks(trainer):
    """The ReLU pattern of each hidden layer in the trainer's last forward."""
    return [trainer.get_activation(l) > 0.0 for l in range(1, len(trainer.dims) - 1)]


def check_mask_flips(masks, pre, x, params, tol=1e-5):
    """Every hidden unit whose FP32 ReLU decision differs from the exact sign
    of its pre-activation must be a near-tie: |z| <= tol * (|a| @ |W| + |b|),
    the accumulated magnitude of the terms summed into z.  Returns the number
    of such flips."""
    flips = 0
    a = np.abs(np.asarray(x, np.float64))
    for l, (mask, z) in enumerate(zip(masks, pre)):
        scale = a @ np.abs(np.asarray(params[2 * l], np.float64)) + \
            np.abs(np.asarray(params[2 * l + 1], np.float64))
        diff = mask != (z > 0.0)
        flips += int(diff.sum())
        if diff.any():
            worst = float(np.max(np.abs(z[diff]) / scale[diff]))
            assert worst <= tol, f"layer {l}: a ReLU decision differs at |z| = {worst:.3g} x scale"
        a = np.where(mask, np.abs(z), 0.0)
    return flips


def argmax_agrees(logits, ref_logits, margin=1e-5):
    """Argmax of every row equal, except rows whose two largest reference
    logits are within margin * max|logit| of each other (a near-tie that any
    correct FP32 order may break either way).  Returns the rows compared."""
    ref = np.asarray(ref_logits, np.float64)
    top2 = np.sort(ref, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > margin * np.abs(ref).max()
    assert np.array_equal(np.argmax(logits, axis=1)[clear], np.argmax(ref, axis=1)[clear])
    return int(clear.sum())
