"""The CUDA-graph step (orca_mlp_graph_capture / _replay).

A captured step replays exactly the ordinary step: after the same number of
steps from the same state, parameters and per-step losses are bit-identical
to ordinary steps -- on the SIMT path (configs[0]'s model) and on the
tensor-core path (single-CTA and cluster-launched CTA-pair kernels, the fused
classifier).  AdamW is refused (its bias corrections change every step), and
the launch counter advances by the captured step's kernel count.
"""
import ctypes

import numpy as np
import pytest

from orcaml_b200.synthetic import init_params, make_batch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from orcaml_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


def _trainer(be, dims, B, path, **kw):
    from orcaml_b200.mlp import MlpTrainer
    tr = MlpTrainer(be, dims, B, optimizer="sgd", gemm_path=path, **kw)
    tr.set_parameters(init_params(dims, 1))
    return tr


@pytest.mark.parametrize("dims,B,path,kw", [
    ([784, 512, 512, 10], 128, "auto", dict(lr=0.1)),
    ([784, 512, 512, 10], 128, "auto", dict(lr=0.01, momentum=0.9)),
    ([784, 1024, 1024, 10], 512, "tc", dict(lr=0.01, momentum=0.9)),
])
def test_graph_replay_equals_ordinary_steps(be, dims, B, path, kw):
    x, t, _ = make_batch(dims, B, 0)
    xs, ts = be.from_f32_slice(list(x.shape), x), be.from_f32_slice(list(t.shape), t)
    eager, graphed = _trainer(be, dims, B, path, **kw), _trainer(be, dims, B, path, **kw)
    le, lg = be.zeros([1]), be.zeros([1])
    eager_losses, graph_losses = [], []
    for _ in range(5):
        eager.step_device(xs.device_ptr, ts.device_ptr, le.device_ptr)
        eager_losses.append(float(be.to_f32_vec(le)[0]))
    graphed.graph_capture(xs.device_ptr, ts.device_ptr, lg.device_ptr)   # runs step 1
    graph_losses.append(float(be.to_f32_vec(lg)[0]))
    n0 = be.launch_count()
    for _ in range(4):
        graphed.graph_step()
        graph_losses.append(float(be.to_f32_vec(lg)[0]))
    per_step = (be.launch_count() - n0) // 4
    assert per_step > 5
    assert graph_losses == eager_losses
    for p, q in zip(eager.get_parameters(), graphed.get_parameters()):
        assert np.array_equal(p, q)
    graphed.graph_release()
    with pytest.raises(ValueError):
        graphed.graph_step()
    eager.close()
    graphed.close()


def test_graph_capture_refuses_adamw(be):
    from orcaml_b200._lib import OrcaError
    from orcaml_b200.mlp import MlpTrainer
    dims, B = [64, 32, 10], 16
    tr = MlpTrainer(be, dims, B, optimizer="adamw", lr=1e-3)
    x, t, _ = make_batch(dims, B, 0)
    xs, ts = be.from_f32_slice(list(x.shape), x), be.from_f32_slice(list(t.shape), t)
    with pytest.raises(OrcaError, match="NOT_IMPLEMENTED"):
        tr.graph_capture(xs.device_ptr, ts.device_ptr)
    tr.close()
