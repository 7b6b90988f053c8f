"""Failure detection on one GPU, without a fault.

Every device-side wait of the library (the GEMM's mbarrier handshakes) is
bounded; when a bound runs out the kernel records DEV_WAIT_TIMEOUT and
returns, and the host call reports ORCA_TIMEOUT with the context still usable.
The self-test kernel runs exactly that wait on an mbarrier nothing completes.
Host-side waits are bounded by the context's deadline (orca_ctx_set_timeout /
orca_ctx_sync); a deadline that passes raises OrcaTimeout and the enqueued
work still completes.  Nothing here traps, faults or hangs the GPU.
"""
import time

import numpy as np
import pytest

from tests.gpu_util import assert_fp32_gemm

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from orcaml_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


@pytest.mark.parametrize("limit", [0.02, 0.2])
def test_device_wait_runs_out_and_context_survives(be, limit):
    from orcaml_b200._lib import OrcaTimeout
    t0 = time.monotonic()
    with pytest.raises(OrcaTimeout, match="bound"):
        be.selftest_wait_timeout(limit)
    el = time.monotonic() - t0
    assert limit <= el < limit + 5.0
    a = np.arange(1000, dtype=np.float32)
    got = be.to_f32_vec(be.add(be.from_f32_slice([1000], a), be.from_f32_slice([1000], a), [1000]))
    assert np.array_equal(got, a + a)
    be.synchronize()                 # the error word was cleared


@pytest.mark.parametrize("limit", [0.0, -1.0, 11.0])
def test_selftest_rejects_bad_limits(be, limit):
    from orcaml_b200._lib import OrcaError
    with pytest.raises(OrcaError, match="ORCA_INVALID_ARGUMENT"):
        be.selftest_wait_timeout(limit)


def test_set_timeout_validation(be):
    from orcaml_b200._lib import OrcaError
    for bad in (0.0, -3.0):
        with pytest.raises(OrcaError, match="ORCA_INVALID_ARGUMENT"):
            be.set_timeout(bad)
    be.set_timeout(600.0)


def test_host_deadline_passes_while_work_completes(be):
    """A sync whose deadline is shorter than the queued work raises
    OrcaTimeout; the work is not lost and a later sync sees it finish."""
    from orcaml_b200._lib import OrcaTimeout
    rng = np.random.default_rng(5)
    m = n = k = 4096
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    sa, sb = be.from_f32_slice([m * k], a), be.from_f32_slice([k * n], b)
    be.synchronize()
    outs = [be.gemm_ex(m, n, k, sa, False, sb, True, 1) for _ in range(4)]   # SIMT: slow on purpose
    with pytest.raises(OrcaTimeout):
        be.synchronize(timeout_s=1e-6)
    be.synchronize()
    rows = slice(0, 64)
    c = be.to_f32_vec(outs[-1]).reshape(m, n)
    assert_fp32_gemm(c[rows], a[rows], b)
