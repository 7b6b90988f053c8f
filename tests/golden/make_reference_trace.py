"""Record the calls the reference's own Python makes into its compiled module.

Run in the development container, where the reference source tree is mounted:

    python tests/golden/make_reference_trace.py /path/to/reference/python

The reference's pure-Python package (python/orca/nn, optim) drives everything
through the compiled module `orca.orca_python` (orca-python/src/lib.rs:
909-919): Tensor factories, arithmetic, autograd (backward, grad, set_grad,
detach), no_grad.  This script installs the restated module of
oracle/orca_shim.py behind a recording proxy, runs the reference's unchanged
Sequential(Linear, ReLU, Linear, ReLU, Linear) + CrossEntropyLoss + SGD on
BASELINE configs[0] (784-512-512-10, batch 128, lr 0.1) for 20 steps
(python/orca/nn/model.py:546-552: zero_grad, forward, loss, backward, step),
and writes every call -- receiver, method, arguments, which result object
came back -- to reference_trace_c0.json.gz.

tests/test_gpu_reference_trace.py replays that call sequence against the
CUDA drop-in (orcaml_b200.orca_python) on a B200, where the reference tree is
not available, and checks the losses the reference's code read back
(loss.to_list()) and its final parameters against the golden c0 fixture.

Data: the weights, inputs and targets come from orcaml_b200.synthetic
(init_params seed 1, make_batch seed 0) and are recorded by name, not value.
"""
from __future__ import annotations

import gzip
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from orcaml_b200.synthetic import CONFIGS, init_params, make_batch  # noqa: E402

STEPS = 20
OUT = os.path.join(HERE, "reference_trace_c0.json.gz")


class Recorder:
    """Proxy factory: wraps the stand-in module's objects and logs calls."""

    def __init__(self, shim, named_arrays):
        self.shim = shim
        self.log = []
        self.ids = {}          # id(inner) -> trace id (objects kept alive in self.keep)
        self.keep = []
        self.named = {}        # data fingerprint -> array name
        for name, arr in named_arrays.items():
            self.named[self._fingerprint(np.asarray(arr, np.float32).reshape(-1))] = name
        rec = self

        class Tensor:                      # the recorded `orca.orca_python.Tensor`
            __slots__ = ("_inner", "_tid", "__weakref__")

            def __init__(self, *a, **k):
                raise TypeError("use the factories")

            # properties (pure queries: recorded so that replay sees the same calls)
            @property
            def shape(self):
                return rec.call(self, "shape", (), {}, prop=True)

            @property
            def dtype(self):
                return rec.call(self, "dtype", (), {}, prop=True)

            @property
            def device(self):
                return rec.call(self, "device", (), {}, prop=True)

            @property
            def requires_grad(self):
                return rec.call(self, "requires_grad", (), {}, prop=True)

            def __repr__(self):
                return f"RecordedTensor#{self._tid}"

        def method(name):
            def f(self, *a, **k):
                return rec.call(self, name, a, k)
            f.__name__ = name
            return f

        def static(name):
            def f(*a, **k):
                return rec.call(None, name, a, k)
            f.__name__ = name
            return staticmethod(f)

        for name in ["zeros", "ones", "scalar", "rand_uniform", "randn", "rand_dropout_mask",
                     "einsum", "from_list"]:
            setattr(Tensor, name, static(name))
        for name in ["to", "to_list", "require_grad", "zero_grad", "backward", "grad", "detach",
                     "set_grad", "to_dtype", "has_nan_or_inf", "expand", "sum_to_shape",
                     "max_to_shape", "reshape", "transpose", "sum", "mean", "relu", "sigmoid",
                     "sqrt", "exp", "log", "__add__", "__radd__", "__sub__", "__rsub__",
                     "__mul__", "__rmul__", "__truediv__", "__rtruediv__", "__neg__",
                     "__matmul__"]:
            setattr(Tensor, name, method(name))
        self.Tensor = Tensor

    @staticmethod
    def _fingerprint(a):
        a = np.ascontiguousarray(a, np.float32)
        return (a.size, float(a[:8].sum()) if a.size else 0.0, hash(a.tobytes()))

    def wrap(self, inner):
        key = id(inner)
        if key in self.ids:
            t = self.ids[key]
            return t
        t = object.__new__(self.Tensor)
        t._inner = inner
        t._tid = len(self.keep)
        self.keep.append((inner, t))
        self.ids[key] = t
        return t

    def enc(self, v, data_arg=False):
        if isinstance(v, self.Tensor):
            return {"t": v._tid}
        if data_arg:
            arr = np.asarray(v, np.float32).reshape(-1)
            name = self.named.get(self._fingerprint(arr))
            if name is not None:
                return {"array": name}
            if arr.size <= 64:
                return {"list": [float(x) for x in arr]}
            raise ValueError(f"unregistered tensor data of {arr.size} values")
        if isinstance(v, (list, tuple)):
            return [self.enc(x) for x in v]
        if isinstance(v, self.shim.DType):
            return {"dtype": repr(v).split(".", 1)[1]}      # F32, F64, ...
        if isinstance(v, self.shim.Device):
            return {"device": v.kind}
        if isinstance(v, (bool, int, float, str)) or v is None:
            return v
        if isinstance(v, (np.floating, np.integer)):
            return v.item()
        raise TypeError(f"cannot record argument {type(v)}")

    def unwrap(self, v):
        if isinstance(v, self.Tensor):
            return v._inner
        if isinstance(v, (list, tuple)):
            return type(v)(self.unwrap(x) for x in v)
        return v

    def call(self, obj, name, args, kwargs, prop=False):
        entry = {"op": name}
        if obj is not None:
            entry["self"] = obj._tid
        data_pos = 0 if name == "from_list" else -1
        entry["args"] = [self.enc(a, data_arg=(i == data_pos)) for i, a in enumerate(args)]
        entry["kwargs"] = {k: self.enc(v, data_arg=(k == "data" and name == "from_list"))
                           for k, v in kwargs.items()}
        target = obj._inner if obj is not None else self.shim.Tensor
        if prop:
            out = getattr(target, name)
        else:
            out = getattr(target, name)(*[self.unwrap(a) for a in args],
                                        **{k: self.unwrap(v) for k, v in kwargs.items()})
        if isinstance(out, self.shim.Tensor):
            out = self.wrap(out)
            entry["out"] = out._tid
        elif name == "to_list" and len(out) <= 16:
            entry["value"] = [float(x) for x in out]
        elif name in ("has_nan_or_inf", "requires_grad"):
            entry["value"] = bool(out)
        elif name == "shape":
            entry["value"] = list(out)
        self.log.append(entry)
        return out

    def module(self):
        import types
        mod = types.ModuleType("orca.orca_python")
        mod.Tensor = self.Tensor
        mod.DType = self.shim.DType
        mod.Device = self.shim.Device
        mod.save_tensors = self.shim.save_tensors
        mod.load_tensors = self.shim.load_tensors
        rec = self

        def set_grad_enabled(enabled):
            rec.log.append({"op": "set_grad_enabled", "args": [bool(enabled)], "kwargs": {}})
            return rec.shim.set_grad_enabled(enabled)

        def is_grad_enabled():
            return rec.shim.is_grad_enabled()

        mod.set_grad_enabled = set_grad_enabled
        mod.is_grad_enabled = is_grad_enabled
        return mod


def main(ref_python: str) -> None:
    from oracle import orca_shim
    cfg = CONFIGS["c0"]
    dims = cfg.dims
    params = init_params(dims, 1)
    x, t, _ = make_batch(dims, cfg.batch, 0)
    named = {f"param{i}": p for i, p in enumerate(params)}
    named.update({"x": x, "t": t})
    rec = Recorder(orca_shim, named)
    sys.modules["orca.orca_python"] = rec.module()
    if ref_python not in sys.path:
        sys.path.insert(0, ref_python)
    import orca  # the reference package, unchanged
    nn = orca.nn
    layers = []
    for i in range(len(dims) - 1):
        layers.append(nn.Linear(dims[i], dims[i + 1]))
        if i + 2 < len(dims):
            layers.append(nn.ReLU())
    model = nn.Sequential(*layers)
    for p, arr in zip(model.parameters(), params):
        p.update(orca.Tensor.from_list(arr.reshape(-1), shape=list(arr.shape), requires_grad=True))
    opt = orca.optim.SGD(model.parameters(), lr=cfg.lr)
    loss_fn = nn.CrossEntropyLoss()
    X = orca.Tensor.from_list(x.reshape(-1), shape=list(x.shape))
    T = orca.Tensor.from_list(t.reshape(-1), shape=list(t.shape))
    losses = []
    for _ in range(STEPS):
        opt.zero_grad()
        loss = loss_fn(model(X), T)
        loss.backward()
        opt.step()
        losses.append(loss.to_list()[0])
    final = [p.tensor._tid for p in model.parameters()]
    doc = {"config": "c0", "dims": dims, "batch": cfg.batch, "lr": cfg.lr, "steps": STEPS,
           "arrays": {"params": "init_params(dims, 1)", "x": "make_batch(dims, 128, 0)[0]",
                      "t": "make_batch(dims, 128, 0)[1]"},
           "final_params": final, "losses": [float(v) for v in losses], "calls": rec.log}
    with gzip.open(OUT, "wt") as f:
        json.dump(doc, f, separators=(",", ":"))
    ops = {}
    for e in rec.log:
        ops[e["op"]] = ops.get(e["op"], 0) + 1
    print(f"wrote {OUT}: {len(rec.log)} calls, {len(rec.keep)} tensors; ops {ops}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference/python")
