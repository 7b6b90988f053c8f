"""The reference's own Python, as a recorded call sequence, on the CUDA drop-in.

The reference's nn/optim package (pure Python) runs on whatever module is
registered as `orca.orca_python` (orca-python/src/lib.rs:909-919).  Its source
tree is not on the GPU box, so tests/golden/make_reference_trace.py ran the
reference's unchanged Sequential(Linear, ReLU, Linear, ReLU, Linear) +
CrossEntropyLoss + SGD (20 steps) in the development
container and recorded every call it made into that module -- 1407 calls:
factories, matmul, expand, the loss's ops, backward, grad/detach/
require_grad, no_grad toggles -- with the receiver, arguments and result of
each.  This test makes the same calls, in the same order, on the drop-in
(orcaml_b200.orca_python, every tensor on the B200) and checks what the
reference's code observed: each step's loss.to_list() within 1e-4 of the
recorded value (which is the golden c0 trace of the reference's Python, bit
for bit) and the final parameters within 1e-4 of the golden c0 fixture.
"""
import gzip
import json
import os

import numpy as np
import pytest

from orcaml_b200.synthetic import init_params, make_batch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _load():
    with gzip.open(os.path.join(HERE, "golden", "reference_trace_c0.json.gz"), "rt") as f:
        return json.load(f)


def test_reference_python_call_sequence_on_the_drop_in(golden):
    from orcaml_b200 import orca_python as op
    doc = _load()
    dims, batch = doc["dims"], doc["batch"]
    params = init_params(dims, 1)
    x, t, _ = make_batch(dims, batch, 0)
    arrays = {f"param{i}": p for i, p in enumerate(params)}
    arrays.update({"x": x, "t": t})
    dtypes = {"F32": op.DType.FLOAT32, "F64": op.DType.FLOAT64}
    objs = {}

    def dec(v, data=False):
        if isinstance(v, dict):
            if "t" in v:
                return objs[v["t"]]
            if "array" in v:
                return arrays[v["array"]].reshape(-1).tolist()
            if "list" in v:
                return v["list"]
            if "dtype" in v:
                return dtypes[v["dtype"]]
            if "device" in v:
                return v["device"]
            raise ValueError(v)
        if isinstance(v, list):
            return [dec(a) for a in v]
        return v

    losses = []
    for i, e in enumerate(doc["calls"]):
        op_name = e["op"]
        if op_name == "set_grad_enabled":
            op.set_grad_enabled(*e["args"])
            continue
        args = [dec(a) for a in e["args"]]
        kwargs = {k: dec(v) for k, v in e["kwargs"].items()}
        if "self" in e:
            target = objs[e["self"]]
            attr = getattr(target, op_name)
            out = attr if op_name in ("shape", "dtype", "device", "requires_grad") else \
                attr(*args, **kwargs)
        else:
            out = getattr(op.Tensor, op_name)(*args, **kwargs)
        if "out" in e:
            assert isinstance(out, op.Tensor), (i, e)
            objs[e["out"]] = out
        if "value" in e:
            if op_name == "to_list":
                assert len(out) == len(e["value"])
                ref = np.float32(e["value"][0])
                assert abs(out[0] - ref) <= 1e-4 * abs(ref), (i, out[0], ref)
                losses.append(out[0])
            else:
                assert out == e["value"], (i, e, out)
    assert len(losses) == doc["steps"]
    # The recorded losses are the reference's own c0 trace.
    ref_losses = [np.frombuffer(bytes.fromhex(h), np.float32)[0]
                  for h in golden["c0"]["loss_bits"][0]]
    assert np.array_equal(np.float32(doc["losses"]), np.float32(ref_losses))
    final = golden["c0"]["final"]
    for j, tid in enumerate(doc["final_params"]):
        p = np.asarray(objs[tid].to_list(), np.float32)
        assert abs(float(p.sum(dtype=np.float64)) - final["sum"][j]) <= \
            1e-4 * final["abs_sum"][j], j
        assert abs(float(np.abs(p).sum(dtype=np.float64)) - final["abs_sum"][j]) <= \
            1e-4 * final["abs_sum"][j], j
        np.testing.assert_allclose(p[:8], final["first8"][j], rtol=1e-3, atol=1e-5)
