"""The CUDA drop-in for `orca.orca_python` (orcaml_b200/orca_python.py).

* The reference's own known-answer autograd tests, run through the drop-in's
  Tensor on the GPU: y = x@w, loss = (y-10)^2 gives dW = [-20, -30]
  (orca-autograd/tests/autograd_tests.rs:6-52); relu([-1, 2]) and its
  gradient (:55-90); d(x^2)/dx = 4 and d(x^3 + 2x^2 + 5x)/dx = 25 at x = 2
  (python/tests/test_api.py:53-61, 196-218); d(x@W)/dW[0] = 1.5 (:250-279).
* A 3-layer MLP with a softmax cross-entropy, composed from Tensor ops exactly
  as a user program would, runs on both the drop-in (GPU) and the oracle's
  Tensor (CPU, the reference's op semantics): loss and every gradient agree
  within 1e-5 relative (the only difference is the GEMM summation order).
* Broadcasting, scalar operands, grad mode, shape errors, dtype casts and
  safetensors round trips.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def op():
    from orcaml_b200 import orca_python
    return orca_python


def test_kat_autograd_matmul(op):
    T = op.Tensor
    x = T.from_list([2.0, 3.0], shape=[1, 2], requires_grad=True)
    w = T.from_list([1.0, 1.0], shape=[2, 1], requires_grad=True)
    diff = x @ w - T.from_list([10.0], shape=[1, 1])
    (diff * diff).backward()
    assert w.grad().to_list() == [-20.0, -30.0]
    assert x.grad().to_list() == [-10.0, -10.0]


def test_kat_relu(op):
    T = op.Tensor
    x = T.from_list([-1.0, 2.0], shape=[1, 2], requires_grad=True)
    y = x.relu()
    assert y.to_list() == [0.0, 2.0]
    (y * T.from_list([1.0, 1.0], shape=[1, 2])).backward()
    assert x.grad().to_list() == [0.0, 1.0]


def test_kat_square_poly_and_linear(op):
    T = op.Tensor
    x = T.from_list([2.0], shape=[1, 1], requires_grad=True)
    (x * x).backward()
    assert x.grad().to_list() == [4.0]
    x = T.from_list([2.0], shape=[1], requires_grad=True)
    (x * x * x + x * x * T.scalar(2.0) + x * T.scalar(5.0)).backward()
    assert abs(x.grad().to_list()[0] - 25.0) < 1e-5
    xi = T.from_list([1.5, -2.0], shape=[1, 2])
    W = T.from_list([0.8, 1.2], shape=[2, 1], requires_grad=True)
    (xi @ W).backward()
    assert W.grad().to_list() == [1.5, -2.0]


def _mlp_program(T, x, t, params, B, C):
    """Linear-ReLU-Linear-ReLU-Linear and a softmax cross-entropy, written with
    the Tensor surface only (works on any implementation of it)."""
    h = x
    n = len(params) // 2
    for i in range(n):
        W, b = params[2 * i], params[2 * i + 1]
        h = h @ W + b
        if i + 1 < n:
            h = h.relu()
    m = h.max_to_shape([B, 1])
    z = h - m
    lse = z.exp().sum_to_shape([B, 1]).log()
    logp = z - lse
    return -((t * logp).sum() * (1.0 / B))


def test_mlp_program_matches_oracle_tensor(op):
    from oracle.orca_shim import Tensor as OracleTensor
    from orcaml_b200.synthetic import init_params, make_batch
    dims, B = [784, 96, 64, 10], 32
    x, t, _ = make_batch(dims, B, 4)
    init = init_params(dims, 1)
    results = []
    for T in (op.Tensor, OracleTensor):
        T_params = [T.from_list(p.reshape(-1), shape=list(p.shape), requires_grad=True)
                    for p in init]
        xt = T.from_list(x.reshape(-1), shape=[B, dims[0]])
        tt = T.from_list(t.reshape(-1), shape=[B, dims[-1]])
        loss = _mlp_program(T, xt, tt, T_params, B, dims[-1])
        loss.backward()
        grads = [np.array(p.grad().to_list(), np.float32) for p in T_params]
        results.append((loss.to_list()[0], grads))
        T_params[0].zero_grad()
    (lg, gg), (lo, go) = results
    assert abs(lg - lo) <= 1e-5 * abs(lo)
    for a, b in zip(gg, go):
        assert np.linalg.norm(a - b) <= 1e-5 * np.linalg.norm(b)


def test_broadcast_scalars_and_errors(op):
    T = op.Tensor
    a = T.from_list(np.arange(6, dtype=np.float32), shape=[2, 3], requires_grad=True)
    b = T.from_list([10.0, 20.0, 30.0], shape=[1, 3], requires_grad=True)
    y = ((a + b) * 2.0 - 1.0) / 4.0 + (1.0 - a) + 3.0 * a
    ref = ((np.arange(6).reshape(2, 3) + [10, 20, 30]) * 2 - 1) / 4 + (1 - np.arange(6).reshape(2, 3)) \
        + 3 * np.arange(6).reshape(2, 3)
    np.testing.assert_allclose(np.array(y.to_list()).reshape(2, 3), ref, rtol=1e-6)
    y.sum().backward()
    np.testing.assert_allclose(a.grad().to_list(), [0.5 - 1 + 3] * 6, rtol=1e-6)
    np.testing.assert_allclose(b.grad().to_list(), [1.0] * 3, rtol=1e-6)   # 2 rows x 0.5
    a.zero_grad()
    with pytest.raises(ValueError):
        T.zeros([2, 3]) + T.zeros([4, 5])
    with pytest.raises(ValueError):
        T.zeros([2, 3]) @ T.zeros([2, 3])
    with pytest.raises(ValueError):
        T.from_list([1.0, 2.0], shape=[3])
    with pytest.raises(ValueError):
        T.zeros([2]).backward()          # does not require grad
    with pytest.raises(ValueError):
        op.Device("tpu")


def test_grad_mode_and_detach(op):
    T = op.Tensor
    x = T.from_list([3.0], shape=[1], requires_grad=True)
    op.set_grad_enabled(False)
    try:
        assert not op.is_grad_enabled()
        y = x * x
        assert not y.requires_grad
    finally:
        op.set_grad_enabled(True)
    z = (x * x).detach()
    assert not z.requires_grad and z.to_list() == [9.0]
    x.zero_grad()


def test_dtype_cast_and_repr(op):
    T = op.Tensor
    a = T.from_list([1.5, -2.25], shape=[2])
    d = a.to_dtype(op.DType.FLOAT64)
    assert d.dtype == op.DType.FLOAT64 and d.to_list() == [1.5, -2.25]
    assert d.to_dtype(op.DType.FLOAT32).to_list() == [1.5, -2.25]
    assert repr(op.DType.FLOAT32) == "orca.F32"
    assert "cuda" in repr(a.device)
    assert not a.has_nan_or_inf()
    assert (a / T.zeros([2])).has_nan_or_inf()


def test_safetensors_roundtrip(op, tmp_path):
    T = op.Tensor
    rng = np.random.default_rng(0)
    w = rng.standard_normal((17, 5)).astype(np.float32)
    tensors = {"layer.weight": T.from_list(w.reshape(-1), shape=[17, 5]),
               "layer.bias": T.from_list([0.5, -1.0, 2.0], shape=[1, 3]),
               "f64": T.from_list([1.0, 2.0], shape=[2]).to_dtype(op.DType.FLOAT64)}
    path = str(tmp_path / "ckpt.safetensors")
    op.save_tensors(path, tensors)
    raw = open(path, "rb").read()
    n = int.from_bytes(raw[:8], "little")
    assert n % 8 == 0 and raw[8:9] == b"{"
    back = op.load_tensors(path)
    assert set(back) == set(tensors)
    assert back["layer.weight"].shape == [17, 5]
    assert np.array_equal(np.array(back["layer.weight"].to_list(), np.float32), w.reshape(-1))
    assert back["layer.bias"].to_list() == [0.5, -1.0, 2.0]
    assert back["f64"].dtype == op.DType.FLOAT64 and back["f64"].to_list() == [1.0, 2.0]
    with pytest.raises(RuntimeError):
        op.load_tensors(str(tmp_path / "missing.safetensors"))
