"""BASELINE configs[1] and configs[4] on one GPU.

* configs[1] (784-4096-4096-10, AdamW lr 1e-3 wd 0.01) with a 128-row batch so
  the oracle finishes in seconds: 2 steps on the auto path (its dW products
  take the CTA-pair tensor-core kernel) -- losses within 1e-4 relative (the
  north-star bar), gradients within 1e-5; see the test for the parameters.
* configs[4] (4096-16384x6-1000, AdamW, N(0,1) inputs, per-rank batch 2048,
  1.43 B parameters, ~30 GB on the device) at full size -- far beyond what the
  oracle can run: the first loss is ln(1000) within 0.05 (near-uniform logits
  from the Kaiming-uniform init), the loss is finite and lower after 3 steps
  on the same batch, and the classifier (C = 1000 > 16) takes the plain
  product path.
"""
import numpy as np
import pytest

from oracle import oracle as O
from orcaml_b200.synthetic import CONFIGS, init_params, make_batch
from tests.gpu_util import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from orcaml_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


def test_c1_reduced_batch_matches_oracle(be):
    """Losses of 2 steps within 1e-4 and the first step's
    gradients within 1e-5 at identical parameters.  Parameters are held to
    1e-3: Adam's first updates are about +-lr per weight whatever the
    gradient's size, so a ReLU pre-activation that two correct FP32 summation
    orders round to opposite signs moves that unit's weights by up to 2 lr --
    the mask-flip sensitivity measured for SGD in
    tests/test_oracle.py::test_oracle_order_sensitivity, amplified by the sign
    normalisation (measured here: 1.9e-4 on W1 after 2 steps).  The AdamW
    arithmetic itself is bit-exact with the oracle
    (test_gpu_primitives.py::test_optimizer_kernels_bit_exact)."""
    from orcaml_b200.mlp import MlpTrainer
    cfg = CONFIGS["c1"]
    B = 128
    kw = dict(lr=cfg.lr, weight_decay=cfg.weight_decay)
    x, t, _ = make_batch(cfg.dims, B, 0)
    g0 = MlpTrainer(be, cfg.dims, B, optimizer="adamw", lr=0.0, weight_decay=0.0)
    g0.set_parameters(init_params(cfg.dims, 1))
    g0.step(x, t)
    _, grads_ref, _ = O.mlp_forward_backward(cfg.dims, init_params(cfg.dims, 1), x, t)
    for i, (g, r) in enumerate(zip(g0.get_grads(), grads_ref)):
        assert rel_err(g, r) <= 1e-5, (i, rel_err(g, r))
    g0.close()
    tr = MlpTrainer(be, cfg.dims, B, optimizer="adamw", **kw)
    tr.set_parameters(init_params(cfg.dims, 1))
    ref = O.OracleTrainer(cfg.dims, init_params(cfg.dims, 1), optimizer="adamw", **kw)
    for step in range(2):
        lg, lr_ = tr.step(x, t), ref.step(x, t)
        assert abs(lg - lr_) <= 1e-4 * abs(lr_), (step, lg, lr_)
    for p, q in zip(tr.get_parameters(), ref.params):
        assert rel_err(p, q) <= 1e-3
    tr.close()


def test_c4_full_size_properties(be):
    from orcaml_b200.mlp import MlpTrainer
    cfg = CONFIGS["c4"]
    assert cfg.n_params == 1_425_769_448
    x, t, _ = make_batch(cfg.dims, cfg.batch, 0, cfg.inputs)
    tr = MlpTrainer(be, cfg.dims, cfg.batch, optimizer="adamw", lr=cfg.lr,
                    weight_decay=cfg.weight_decay)
    tr.set_parameters(init_params(cfg.dims, 1))
    losses = [tr.step(x, t) for _ in range(3)]
    assert all(np.isfinite(losses))
    assert abs(losses[0] - np.log(1000.0)) < 0.05
    assert losses[2] < losses[0]
    tr.close()
