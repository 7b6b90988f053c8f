"""FP32-accuracy of the GEMM paths, through orca_gemm_ex / orca_matmul / orca_linear_fwd.

Every operand orientation the MLP step uses (X@W: A K-major, B MN-major;
X^T@dY: both MN-major; dY@W^T: both K-major) is checked on the tcgen05
3xTF32 path and on the SIMT path against a float64 product, including
ragged M/N/K tails (K = 784, N = 1000, M = 100) that exercise TMA
out-of-bounds fill and the epilogue's edge masks.
"""
import numpy as np
import pytest

from tests.gpu_util import assert_fp32_gemm

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(3)


@pytest.fixture(scope="module")
def be():
    from orcaml_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


def run(be, m, n, k, a_mn, b_mn, path, scale=1.0):
    a = (RNG.standard_normal((k, m) if a_mn else (m, k)) * scale).astype(np.float32)
    b = (RNG.standard_normal((k, n) if b_mn else (n, k)) * scale).astype(np.float32)
    sa = be.from_f32_slice([a.size], a)
    sb = be.from_f32_slice([b.size], b)
    c = be.to_f32_vec(be.gemm_ex(m, n, k, sa, a_mn, sb, b_mn, path)).reshape(m, n)
    A = a.T if a_mn else a
    B = b if b_mn else b.T
    return c, A, B


SHAPES = [(128, 256, 16), (256, 512, 64), (384, 768, 784), (100, 1000, 200), (1000, 300, 48),
          (520, 260, 4096)]


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True), (False, False), (True, False)])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_tcgen05_orientations(be, m, n, k, a_mn, b_mn):
    c, A, B = run(be, m, n, k, a_mn, b_mn, path=2)
    assert_fp32_gemm(c, A, B)


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True), (False, False)])
@pytest.mark.parametrize("m,n,k", [(37, 53, 29), (4096, 10, 512), (64, 10, 4096), (300, 200, 10),
                                   (128, 128, 128)])
def test_simt_and_skinny(be, m, n, k, a_mn, b_mn):
    c, A, B = run(be, m, n, k, a_mn, b_mn, path=1)
    assert_fp32_gemm(c, A, B)


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True), (False, False), (True, False)])
@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (512, 768, 784), (300, 1000, 200),
                                   (100, 256, 48), (1000, 300, 4096)])
def test_tcgen05_cta_pair_kernel(be, m, n, k, a_mn, b_mn):
    """The two-CTA kernel (256 x 256 tiles, cta_group::2): every orientation,
    ragged M (an odd CTA whose rows all lie past M), ragged N and K."""
    c, A, B = run(be, m, n, k, a_mn, b_mn, path=4)
    assert_fp32_gemm(c, A, B)


@pytest.mark.parametrize("m,n,k", [(512, 512, 256), (384, 768, 784)])
def test_tcgen05_single_cta_kernel_forced(be, m, n, k):
    c, A, B = run(be, m, n, k, False, True, path=3)
    assert_fp32_gemm(c, A, B)


def test_tcgen05_pair_large_tiles_and_waves(be):
    # More pair tiles than clusters: the persistent loop wraps on both CTAs.
    c, A, B = run(be, 4096, 4096, 512, True, True, path=4)
    assert_fp32_gemm(c, A, B)


def test_tcgen05_is_not_plain_tf32(be):
    """A TF32-only product misses the FP32 bound by a wide margin; the
    split path meets it -- evidence that the lo planes are being used."""
    c, A, B = run(be, 256, 256, 1024, False, True, path=2)
    assert_fp32_gemm(c, A, B)
    t32 = lambda x: (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    c_tf32 = (t32(A).astype(np.float64) @ t32(B).astype(np.float64)).astype(np.float32)
    with pytest.raises(AssertionError):
        assert_fp32_gemm(c_tf32, A, B)


def test_tcgen05_large_tiles_and_waves(be):
    # More tiles than SMs (persistent scheduler wraps), both accumulators reused.
    c, A, B = run(be, 2048, 4096, 256, False, True, path=2)
    assert_fp32_gemm(c, A, B)


def test_path_rejects_ineligible(be):
    from orcaml_b200._lib import OrcaError
    with pytest.raises(OrcaError):
        run(be, 32, 32, 8, False, True, path=2)   # too small for the tensor-core tile


def test_matmul_trait_method_batched(be):
    a = RNG.standard_normal((3, 130, 96)).astype(np.float32)
    b = RNG.standard_normal((3, 96, 200)).astype(np.float32)
    c = be.to_f32_vec(be.matmul(be.from_f32_slice([3, 130, 96], a),
                                be.from_f32_slice([3, 96, 200], b),
                                [3, 130, 96], [3, 96, 200])).reshape(3, 130, 200)
    for i in range(3):
        assert_fp32_gemm(c[i], a[i], b[i])


def test_linear_fwd_bias_relu(be):
    m, k, n = 300, 784, 512
    x = RNG.random((m, k), dtype=np.float32)
    w = (RNG.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    bias = (RNG.uniform(-1, 1, (1, n)) / np.sqrt(k)).astype(np.float32)
    out = be.to_f32_vec(be.linear_fwd(be.from_f32_slice([m, k], x), be.from_f32_slice([k, n], w),
                                      be.from_f32_slice([1, n], bias), m, k, n, relu=True))
    z = x.astype(np.float64) @ w.astype(np.float64) + bias
    ref = np.maximum(z, 0)
    scale = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64) + np.abs(bias)
    assert np.all(np.abs(out.reshape(m, n) - ref) <= 1e-5 * scale + 1e-30)


@pytest.mark.parametrize("m,k,n,with_mask", [(300, 784, 512, True), (64, 100, 10, True),
                                             (2048, 512, 1024, False), (7, 5, 3, True)])
def test_linear_bwd_fused(be, m, k, n, with_mask):
    """orca_linear_bwd: dW = x^T dy, db = row sum of dy, dX = dy W^T masked by
    mask > 0, against float64 (FP32-accuracy bound of each product)."""
    x = RNG.standard_normal((m, k)).astype(np.float32)
    w = (RNG.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    dy = RNG.standard_normal((m, n)).astype(np.float32)
    mask = RNG.standard_normal((m, k)).astype(np.float32) if with_mask else None
    up = lambda a: be.from_f32_slice([a.size], a)
    dx, dw, db = be.linear_bwd(up(x), up(w), up(dy), m, k, n,
                               mask=up(mask) if with_mask else None)
    assert_fp32_gemm(be.to_f32_vec(dw).reshape(k, n), x.T, dy)
    ref_db = dy.astype(np.float64).sum(axis=0)
    assert np.all(np.abs(be.to_f32_vec(db) - ref_db) <= 1e-5 * np.abs(dy).astype(np.float64).sum(0))
    got_dx = be.to_f32_vec(dx).reshape(m, k)
    ref = dy.astype(np.float64) @ w.astype(np.float64).T
    scale = np.abs(dy).astype(np.float64) @ np.abs(w).astype(np.float64).T
    if with_mask:
        keep = mask > 0
        assert np.all(got_dx[~keep] == 0)
        assert np.all(np.abs(got_dx - ref)[keep] <= 1e-5 * scale[keep] + 1e-30)
    else:
        assert np.all(np.abs(got_dx - ref) <= 1e-5 * scale + 1e-30)
    _, dw2, _ = be.linear_bwd(up(x), up(w), up(dy), m, k, n, need_dx=False)
    assert np.array_equal(be.to_f32_vec(dw2), be.to_f32_vec(dw))


@pytest.mark.parametrize("k,mean_bound", [(8192, 2.5e-8), (784, 3.5e-8)])
def test_tcgen05_mean_error_at_fp32_level(be, k, mean_bound):
    """The chunked accumulation keeps the tensor-core product at FP32 accuracy
    on the data the step multiplies (ReLU activations x Kaiming-scaled
    weights): mean |C - exact| / sum|a*b| within 1.25x (K = 8192) and 1.75x
    (K = 784) of a serial k-ascending FP32 sum (about 2e-8 here)."""
    rng = np.random.default_rng(7)
    m = n = 256
    a = np.maximum(rng.standard_normal((m, k)), 0).astype(np.float32)
    b = (rng.standard_normal((k, n)) * np.sqrt(2.0 / k)).astype(np.float32)
    sa = be.from_f32_slice([a.size], a)
    sb = be.from_f32_slice([b.size], b)
    c = be.to_f32_vec(be.gemm_ex(m, n, k, sa, False, sb, True, 2)).reshape(m, n)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)
    rel = np.abs(c.astype(np.float64) - exact) / scale
    assert float(rel.mean()) <= mean_bound, float(rel.mean())
