"""The input pipeline on the device (orca_mlp_stage_batch / _step_staged,
orcaml_b200.dataloader.StagedFeeder).

* Staged steps are the ordinary step: training from a DataLoader through the
  feeder (page-locked ring, copy of batch k+1 during step k) gives per-step
  losses and final parameters bit-identical to MlpTrainer.step on the same
  batches -- SIMT and tensor-core shapes, SGD-momentum and AdamW.
* Page-locked and pageable staging give the same result; a slot is consumed
  by one step; out-of-range slots and empty slots are refused with
  ORCA_INVALID_ARGUMENT; restaging a slot replaces its batch.
* The DataLoader's tensors (the drop-in's) hold the collated batch.
"""
import numpy as np
import pytest

from orcaml_b200.synthetic import init_params

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from orcaml_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


def _trainer(be, dims, B, path, opt, kw):
    from orcaml_b200.mlp import MlpTrainer
    tr = MlpTrainer(be, dims, B, optimizer=opt, gemm_path=path, **kw)
    tr.set_parameters(init_params(dims, 1))
    return tr


def _data(dims, n, seed):
    rng = np.random.default_rng(seed)
    X = rng.random((n, dims[0]), dtype=np.float32)
    y = rng.integers(0, dims[-1], n)
    return X, y


@pytest.mark.parametrize("dims,B,path,opt,kw", [
    ([784, 512, 512, 10], 128, "auto", "sgd", dict(lr=0.01, momentum=0.9)),
    ([784, 1024, 1024, 10], 512, "tc", "sgd", dict(lr=0.01, momentum=0.9)),
    ([784, 1024, 1024, 10], 512, "tc", "adamw", dict(lr=1e-3, weight_decay=0.01)),
])
def test_feeder_equals_ordinary_steps(be, dims, B, path, opt, kw):
    from orcaml_b200.dataloader import ArrayDataset, DataLoader, StagedFeeder
    X, y = _data(dims, 7 * B, 3)
    loader = DataLoader(ArrayDataset(X, y, one_hot_classes=dims[-1]), batch_size=B,
                        shuffle=True, seed=5)
    plain, fed = _trainer(be, dims, B, path, opt, kw), _trainer(be, dims, B, path, opt, kw)
    want = [plain.step(x, t) for x, t in loader.numpy_batches()]
    got = StagedFeeder(fed, loader).run()
    assert got == want
    for p, q in zip(plain.get_parameters(), fed.get_parameters()):
        assert np.array_equal(p, q)


def test_stage_slots_pinned_pageable_and_errors(be):
    from orcaml_b200._lib import OrcaError
    from orcaml_b200.dataloader import pinned_empty
    dims, B = [784, 256, 10], 64
    X, y = _data(dims, 3 * B, 8)
    T = np.eye(dims[-1], dtype=np.float32)[y]
    ref = _trainer(be, dims, B, "auto", "sgd", dict(lr=0.05))
    want = [ref.step(X[i * B:(i + 1) * B], T[i * B:(i + 1) * B]) for i in range(3)]

    tr = _trainer(be, dims, B, "auto", "sgd", dict(lr=0.05))
    xp, tp = pinned_empty((B, dims[0])), pinned_empty((B, dims[-1]))
    xp[:], tp[:] = X[:B], T[:B]
    tr.stage_batch(1, xp, tp)                              # page-locked
    tr.stage_batch(0, X[B:2 * B].copy(), T[B:2 * B].copy())   # pageable
    got = [tr.step_staged(1), tr.step_staged(0)]
    with pytest.raises(OrcaError, match="no staged batch"):
        tr.step_staged(0)                                  # consumed
    with pytest.raises(OrcaError):
        tr.step_staged(2)
    with pytest.raises(OrcaError):
        tr.stage_batch(-1, X[:B], T[:B])
    tr.stage_batch(1, X[:B], T[:B])                        # replaced before its step:
    tr.stage_batch(1, X[2 * B:], T[2 * B:])
    got.append(tr.step_staged(1))
    assert got == want
    for p, q in zip(ref.get_parameters(), tr.get_parameters()):
        assert np.array_equal(p, q)


def test_loader_yields_device_tensors(be):
    from orcaml_b200.dataloader import from_arrays
    loader = from_arrays([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]], [0, 1, 2], batch_size=2,
                         one_hot_classes=3)
    xb, tb = next(iter(loader))
    assert xb.shape == [2, 2] and tb.shape == [2, 3]
    assert xb.to_list() == [1.0, 2.0, 3.0, 4.0]
    assert tb.to_list() == [1.0, 0.0, 0.0, 0.0, 1.0, 0.0]
