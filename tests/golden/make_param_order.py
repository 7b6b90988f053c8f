"""Record the reference's Module.parameters() order for MLPs (param_order.json).

Run in the development container, where the reference source tree is mounted:

    python tests/golden/make_param_order.py /path/to/reference/python

Builds the reference's own Sequential(Linear, ReLU, ..., Linear)
(python/orca/nn/container.py, linear.py) on the restated compiled module
(oracle/orca_shim.py) and writes, for each model, the shapes that
model.parameters() yields in order (python/orca/nn/module.py:32-44).  The
gradient arena of the step runner and its exchange plan are checked against
this order by tests/test_bucket_plan_cpu.py.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

# configs[0]'s model, a ragged one, and one with configs[4]'s depth (seven
# Linear layers) at small widths: the order is structural (per Linear its
# weight, then its bias; Linears in Sequential order), so small widths pin it.
MODELS = [[784, 512, 512, 10], [13, 7, 5, 3], [64] + [48] * 6 + [10]]


def main(ref_python: str) -> None:
    from oracle import orca_shim
    orca = orca_shim.install(ref_python)
    nn = orca.nn
    out = []
    for dims in MODELS:
        layers = []
        for i in range(len(dims) - 1):
            layers.append(nn.Linear(dims[i], dims[i + 1]))
            if i + 2 < len(dims):
                layers.append(nn.ReLU())
        model = nn.Sequential(*layers)
        shapes = [list(p.tensor.shape) for p in model.parameters()]
        out.append({"dims": dims, "parameter_shapes": shapes})
    with open(os.path.join(HERE, "param_order.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "param_order.json"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference/python")
