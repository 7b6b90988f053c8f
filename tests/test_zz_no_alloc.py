"""The allocation-free softmax cross-entropy entry point.

orca_softmax_ce_fwd_bwd_noalloc serves callers that cannot allocate device
memory mid-run -- code whose memory belongs to another allocator (a
framework's caching pool, a preallocated arena) or a latency-bound loop where
an allocation could synchronise the GPU.  It takes caller-owned device buffers
for every input and output and keeps its per-row scratch in a fixed device
array whose address the context looked up when it was created.  This file is
collected last so that a failure here, in a run that stops at the first
failure, comes after every other test has run.

Checked through the C ABI: two calls in a row (different batch sizes, so the
shared scratch is reused) give the same loss and gradient as the allocating
entry point and as the oracle's restatement of the reference's loss, within
the tolerance of the other CE tests; the forward-only form (dlogits = NULL)
gives the same loss; a batch above the scratch capacity is refused before
anything is launched.
"""
import ctypes

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


def _problem(rng, batch, classes):
    p = (rng.standard_normal((batch, classes)) * 3).astype(np.float32)
    t = np.zeros((batch, classes), np.float32)
    t[np.arange(batch), rng.integers(0, classes, batch)] = 1.0
    return p, t


def _noalloc(be, ps, ts, batch, classes, loss_buf, dp_buf):
    from orcaml_b200 import _lib as L
    dp = ctypes.c_void_p(dp_buf.device_ptr) if dp_buf is not None else None
    L.check(L.load().orca_softmax_ce_fwd_bwd_noalloc(
        be.ctx, ctypes.c_void_p(ps.device_ptr), ctypes.c_void_p(ts.device_ptr), batch, classes,
        ctypes.c_void_p(loss_buf.device_ptr), dp))


def test_noalloc_matches_allocating_entry_point_and_oracle_twice(be):
    rng = np.random.default_rng(11)
    for batch, classes in [(4096, 10), (1000, 1000)]:          # two calls in a row
        p, t = _problem(rng, batch, classes)
        ps = be.from_f32_slice([batch, classes], p)
        ts = be.from_f32_slice([batch, classes], t)
        ref_loss_s, ref_dp_s = be.softmax_ce_fwd_bwd(ps, ts, batch, classes)
        loss_buf = be.zeros([1])
        dp_buf = be.zeros([batch, classes])
        _noalloc(be, ps, ts, batch, classes, loss_buf, dp_buf)
        ref_loss = be.to_f32_vec(ref_loss_s)[0]
        loss = be.to_f32_vec(loss_buf)[0]
        dp = be.to_f32_vec(dp_buf)
        assert abs(loss - ref_loss) <= 1e-5 * abs(ref_loss)
        np.testing.assert_allclose(dp, be.to_f32_vec(ref_dp_s), rtol=1e-5, atol=1e-9)
        o_loss, o_dp = O.softmax_ce(p, t)
        assert abs(loss - o_loss) <= 1e-5 * abs(o_loss)
        np.testing.assert_allclose(dp.reshape(batch, classes), o_dp, rtol=1e-5, atol=1e-9)


def test_noalloc_forward_only_form(be):
    rng = np.random.default_rng(12)
    batch, classes = 777, 10
    p, t = _problem(rng, batch, classes)
    ps = be.from_f32_slice([batch, classes], p)
    ts = be.from_f32_slice([batch, classes], t)
    loss_buf = be.zeros([1])
    _noalloc(be, ps, ts, batch, classes, loss_buf, None)
    o_loss, _ = O.softmax_ce(p, t, with_grad=False)
    assert abs(be.to_f32_vec(loss_buf)[0] - o_loss) <= 1e-5 * abs(o_loss)


def test_noalloc_rejects_batch_beyond_scratch(be):
    from orcaml_b200._lib import OrcaError
    big = (1 << 20) + 1
    dummy = be.zeros([4])
    with pytest.raises(OrcaError, match="exceeds"):
        _noalloc(be, dummy, dummy, big, 1, dummy, dummy)
