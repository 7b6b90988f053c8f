"""Backend-trait primitives on the GPU vs the CPU oracle, through the C ABI.

Element-wise f32 ops and the serial-order reductions are bit-exact with the
reference CPU backend; exp/log/sigmoid call CUDA's expf/logf, which are within
2 ulp of glibc's, so they are compared at 4 ulp.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from orcaml_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


def up(be, a):
    a = np.ascontiguousarray(a, np.float32)
    return be.from_f32_slice(list(a.shape), a)


def down(be, s, shape):
    return be.to_f32_vec(s).reshape(shape)


RNG = np.random.default_rng(7)


@pytest.mark.parametrize("n", [1, 7, 1000, 65537])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "relu_backward", "exp_backward",
                                "log_backward", "sqrt_backward", "div_backward_lhs",
                                "sigmoid_backward"])
def test_binary_bit_exact(be, op, n):
    a = RNG.standard_normal(n).astype(np.float32)
    b = RNG.standard_normal(n).astype(np.float32)
    if op in ("div", "log_backward", "div_backward_lhs", "sqrt_backward"):
        b = np.where(np.abs(b) < 1e-3, 1.0, b).astype(np.float32)
    got = down(be, getattr(be, op)(up(be, a), up(be, b), [n]), (n,))
    want = getattr(O, op)(a, b)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)) or np.array_equal(got, want)


@pytest.mark.parametrize("op", ["relu", "sqrt"])
def test_unary_bit_exact(be, op):
    a = RNG.standard_normal(4099).astype(np.float32)
    if op == "sqrt":
        a = np.abs(a)
    got = down(be, getattr(be, op)(up(be, a), [4099]), (4099,))
    assert np.array_equal(got, getattr(O, op)(a))


def ulps(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    return np.abs(ai - bi)


@pytest.mark.parametrize("op", ["exp", "log", "sigmoid"])
def test_transcendental_within_4_ulp(be, op):
    a = (RNG.standard_normal(10000) * 4).astype(np.float32)
    if op == "log":
        a = np.concatenate([np.abs(a), np.array([0.0, -1.0, 1e-9], np.float32)])  # clamp path
    got = down(be, getattr(be, op)(up(be, a), [a.size]), (a.size,))
    want = getattr(O, op)(a)
    assert int(ulps(got, want).max()) <= 4


def test_mul_scalar_bit_exact(be):
    a = RNG.standard_normal(5000).astype(np.float32)
    got = down(be, be.mul_scalar(up(be, a), 0.1, [5000]), (5000,))
    assert np.array_equal(got, O.mul_scalar(a, 0.1))


@pytest.mark.parametrize("in_shape,out_shape", [([1, 7], [5, 7]), ([3, 1], [3, 4]),
                                                ([1], [2, 3]), ([2, 1, 3], [2, 4, 3]),
                                                ([4, 5], [4, 5])])
def test_expand(be, in_shape, out_shape):
    a = RNG.standard_normal(int(np.prod(in_shape))).astype(np.float32).reshape(in_shape)
    got = down(be, be.expand(up(be, a), in_shape, out_shape), out_shape)
    assert np.array_equal(got, O.expand(a, in_shape, out_shape))


@pytest.mark.parametrize("in_shape,out_shape", [([4096, 37], [1, 37]), ([9, 10], [9, 1]),
                                                ([5, 6], [1]), ([2, 3, 4], [3, 1]),
                                                ([2, 3, 4], [1, 3, 4]), ([6, 7], [6, 7])])
def test_sum_to_shape_serial_order_bit_exact(be, in_shape, out_shape):
    a = (RNG.standard_normal(int(np.prod(in_shape))) * 10).astype(np.float32).reshape(in_shape)
    got = down(be, be.sum_to_shape(up(be, a), in_shape, out_shape), out_shape)
    assert np.array_equal(got, O.sum_to_shape(a, in_shape, out_shape))


@pytest.mark.parametrize("in_shape,out_shape", [([64, 10], [64, 1]), ([3, 4], [1, 4]),
                                                ([2, 3, 4], [2, 1, 1])])
def test_max_to_shape_and_backward(be, in_shape, out_shape):
    a = RNG.integers(-3, 3, int(np.prod(in_shape))).astype(np.float32).reshape(in_shape)  # ties
    m = down(be, be.max_to_shape(up(be, a), in_shape, out_shape), out_shape)
    assert np.array_equal(m, O.max_to_shape(a, in_shape, out_shape))
    g = RNG.standard_normal(int(np.prod(out_shape))).astype(np.float32).reshape(out_shape)
    gi = down(be, be.max_to_shape_backward(up(be, g), up(be, a), up(be, m), in_shape, out_shape),
              in_shape)
    assert np.array_equal(gi, O.max_to_shape_backward(g, a, m, in_shape, out_shape))


@pytest.mark.parametrize("shape,d0,d1", [([7, 13], 0, 1), ([2, 3, 4], 0, 2), ([5, 1, 6], 1, 2)])
def test_transpose(be, shape, d0, d1):
    a = RNG.standard_normal(int(np.prod(shape))).astype(np.float32).reshape(shape)
    got = be.to_f32_vec(be.transpose(up(be, a), shape, d0, d1))
    assert np.array_equal(got, O.transpose(a, shape, d0, d1).reshape(-1))


def test_accumulate_grad_and_errors(be):
    from orcaml_b200._lib import OrcaError
    a = RNG.standard_normal(100).astype(np.float32)
    b = RNG.standard_normal(100).astype(np.float32)
    got = be.to_f32_vec(be.accumulate_grad(up(be, a), up(be, b)))
    assert np.array_equal(got, O.accumulate_grad(a, b))
    with pytest.raises(OrcaError):
        be.add(up(be, a), up(be, b[:50]), [100])          # shape mismatch -> ValueError
    with pytest.raises(ValueError):
        be.matmul(up(be, a), up(be, b), [10, 10], [9, 10])  # inner dims
    with pytest.raises(ValueError):
        be.transpose(up(be, a), [10, 10], 0, 2)


def test_cast_roundtrip_and_nonfinite(be):
    from orcaml_b200.backend import F16, F32, F64
    a = RNG.standard_normal(33).astype(np.float32)
    s = up(be, a)
    d = be.cast(s, [33], F32, F64)
    back = be.to_f32_vec(be.cast(d, [33], F64, F32))
    assert np.array_equal(back, a)
    h = be.cast(s, [33], F32, F16)
    assert np.array_equal(be.to_f32_vec(be.cast(h, [33], F16, F32)),
                          a.astype(np.float16).astype(np.float32))
    assert not be.has_nan_or_inf(s)
    assert be.has_nan_or_inf(up(be, np.array([1.0, np.inf], np.float32)))


def test_softmax_ce_matches_oracle_including_ties(be, golden):
    case = golden["ce_ties"]
    P = np.array(case["P"], np.float32)
    T = np.array(case["T"], np.float32)
    loss_s, dp_s = be.softmax_ce_fwd_bwd(up(be, P), up(be, T), 4, 4)
    loss = be.to_f32_vec(loss_s)[0]
    dp = be.to_f32_vec(dp_s).reshape(4, 4)
    ref_loss, ref_dp = O.softmax_ce(P, T)
    assert abs(loss - ref_loss) <= 4e-7 * max(1.0, abs(ref_loss))
    np.testing.assert_allclose(dp, ref_dp, rtol=1e-5, atol=1e-7)


def test_softmax_ce_large_batch(be):
    P = (RNG.standard_normal((4096, 10)) * 3).astype(np.float32)
    lab = RNG.integers(0, 10, 4096)
    T = np.zeros((4096, 10), np.float32)
    T[np.arange(4096), lab] = 1
    loss_s, dp_s = be.softmax_ce_fwd_bwd(up(be, P), up(be, T), 4096, 10)
    ref_loss, ref_dp = O.softmax_ce(P, T)
    assert abs(be.to_f32_vec(loss_s)[0] - ref_loss) <= 1e-5 * abs(ref_loss)
    np.testing.assert_allclose(be.to_f32_vec(dp_s).reshape(4096, 10), ref_dp, rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("B,C", [(2048, 1000), (3, 33), (37, 100), (5, 4099), (9, 8192)])
def test_softmax_ce_wide_rows_match_oracle(be, B, C):
    """Rows wider than 32 classes take the warp-per-row kernel (configs[4]'s
    C = 1000 among them): the same serial sums as the reference, so the loss
    and dP agree with the oracle up to expf/logf's ulps; rows with tied
    maxima exercise MaxToShapeBackward's tie rule."""
    P = (RNG.standard_normal((B, C)) * 3).astype(np.float32)
    P[0, : min(C, 4)] = P[0].max() + 1.0          # a four-way tie at the maximum
    T = np.zeros((B, C), np.float32)
    T[np.arange(B), RNG.integers(0, C, B)] = 1.0
    T[-1] = 1.0 / C                                # a soft target row
    loss_s, dp_s = be.softmax_ce_fwd_bwd(up(be, P), up(be, T), B, C)
    ref_loss, ref_dp = O.softmax_ce(P, T)
    assert abs(be.to_f32_vec(loss_s)[0] - ref_loss) <= 1e-5 * abs(ref_loss)
    np.testing.assert_allclose(down(be, dp_s, (B, C)), ref_dp, rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("opt", ["sgd", "sgdm", "sgdm_wd_damp", "adamw"])
def test_optimizer_kernels_bit_exact(be, opt):
    n = 10007
    p = RNG.standard_normal(n).astype(np.float32)
    g = RNG.standard_normal(n).astype(np.float32)
    ps, gs = up(be, p), up(be, g)
    pr = p.copy()
    if opt == "adamw":
        m = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        ms, vs = up(be, m), up(be, v)
        for t in (1, 2, 3):
            be.adamw_step(ps, gs, ms, vs, 1e-3, 0.9, 0.999, 1e-8, 0.01, t)
            O.adamw_step(pr, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, t)
        assert np.array_equal(be.to_f32_vec(ms), m)
        assert np.array_equal(be.to_f32_vec(vs), v)
    else:
        mom = 0.0 if opt == "sgd" else 0.9
        wd, damp = (0.01, 0.1) if opt == "sgdm_wd_damp" else (0.0, 0.0)
        v = np.zeros(n, np.float32)
        vs = up(be, v)
        for i in range(3):
            be.sgd_step(ps, gs, vs if mom else None, 0.01, mom, damp, wd, first=(i == 0))
            O.sgd_step(pr, g, v if mom else None, 0.01, mom, damp, wd, first=(i == 0))
    assert np.array_equal(be.to_f32_vec(ps), pr)
