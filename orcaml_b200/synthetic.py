"""Seeded synthetic MLP problems with the shapes of the north-star configs.

The reference seeds nothing (orca-tensor/src/tensor.rs:63 draws weights from an
unseeded thread_rng), so every harness here creates the initial tensors itself
and injects them, the way python/tests/test_phase8.py:115-116 injects fixed
weights through Tensor.from_list:

* weights: Kaiming-uniform with a = sqrt(5) over fan_in = in_features
  (python/orca/nn/init.py:84-101 -> bound = 1/sqrt(in)), bias uniform in the
  same bound (python/orca/nn/linear.py:34-36); drawn from
  numpy default_rng(weight_seed), layer by layer, W then b (Module.parameters()
  order, python/orca/nn/module.py:32-44), identical on every rank;
* inputs: default_rng(rank).random((B, D0), float32) in [0, 1) (or N(0,1) for
  the deep config), then labels default_rng(rank).integers(0, C, B) from the
  same generator, one-hot encoded as the reference's CrossEntropyLoss expects
  (python/orca/nn/loss.py:64-72).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Sequence

import numpy as np


@dataclass
class MlpConfig:
    name: str
    dims: List[int]
    batch: int                    # per rank
    optimizer: str                # "sgd" | "adamw"
    lr: float
    momentum: float = 0.0
    dampening: float = 0.0
    weight_decay: float = 0.0
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    inputs: str = "uniform"       # "uniform" | "normal"
    world: List[int] = field(default_factory=lambda: [1])

    @property
    def n_params(self) -> int:
        return sum(self.dims[i] * self.dims[i + 1] + self.dims[i + 1]
                   for i in range(len(self.dims) - 1))

    def flops_per_sample(self) -> int:
        """GEMM FLOPs per sample of one step: forward 2*K*N per layer, dW the
        same, dX for every layer but the first (no input gradient)."""
        f = 0
        for i in range(len(self.dims) - 1):
            k, n = self.dims[i], self.dims[i + 1]
            f += 2 * k * n * (3 if i > 0 else 2)
        return f


# BASELINE.json configs[0..4] (c3 is the all-reduce sweep, not an MLP).
CONFIGS = {
    "c0": MlpConfig("c0", [784, 512, 512, 10], 128, "sgd", 0.1),
    "c1": MlpConfig("c1", [784, 4096, 4096, 10], 1024, "adamw", 1e-3, weight_decay=0.01,
                    world=[2]),
    "c2": MlpConfig("c2", [784, 8192, 8192, 10], 4096, "sgd", 0.01, momentum=0.9,
                    world=[1, 2, 4, 8]),
    "c4": MlpConfig("c4", [4096] + [16384] * 6 + [1000], 2048, "adamw", 1e-3, weight_decay=0.01,
                    inputs="normal", world=[8]),
}


def init_params(dims: Sequence[int], seed: int = 1) -> List[np.ndarray]:
    rng = np.random.default_rng(seed)
    params = []
    for i in range(len(dims) - 1):
        fan_in, fan_out = dims[i], dims[i + 1]
        bound = 1.0 / np.sqrt(fan_in)
        w = rng.uniform(-bound, bound, size=(fan_in, fan_out)).astype(np.float32)
        b = rng.uniform(-bound, bound, size=(1, fan_out)).astype(np.float32)
        params += [w, b]
    return params


def make_batch(dims: Sequence[int], batch: int, rank: int = 0, inputs: str = "uniform"):
    rng = np.random.default_rng(rank)
    if inputs == "uniform":
        x = rng.random((batch, dims[0]), dtype=np.float32)
    else:
        x = rng.standard_normal((batch, dims[0]), dtype=np.float32)
    labels = rng.integers(0, dims[-1], batch)
    t = np.zeros((batch, dims[-1]), dtype=np.float32)
    t[np.arange(batch), labels] = 1.0
    return x, t, labels.astype(np.int32)
