"""A CPU stand-in for the reference's compiled `orca.orca_python` module.

TEST INFRASTRUCTURE ONLY.  The reference's Python frontend (python/orca/**:
nn, optim, distributed, ...) is pure Python over one compiled PyO3 module,
`orca.orca_python` (orca-python/src/lib.rs:909-919), which cannot be built
here (no Rust toolchain).  This module provides the same surface, built from

  * a restated tape autograd -- orca-autograd/src/backend.rs (op wrappers
    74-1281, backward nodes 1283-1930) and tape.rs (reverse sweep over every
    recorded node, grads accumulated existing + new); and
  * the restated CPU backend primitives of oracle/orca_oracle.c
    (orca-backend-cpu/src/backend.rs).

so that the reference's own Python code (Sequential/Linear/ReLU/
CrossEntropyLoss/SGD/AdamW/DistributedDataParallel) runs unchanged on top of
it.  tests/golden/make_golden.py uses this in the development container to
turn the reference's own Python into golden vectors; nothing on the GPU box
imports it.

Only FP32 is supported (the north-star path is FP32); other dtypes raise.
"""
from __future__ import annotations

import math
import sys
import threading
from typing import List, Optional

import numpy as np

from . import oracle as O

# ---------------------------------------------------------------- dtype/device
class DType:
    """orca.DType (orca-python/src/lib.rs:42-81)."""

    def __init__(self, name: str):
        self._name = name

    def __eq__(self, other):
        return isinstance(other, DType) and other._name == self._name

    def __ne__(self, other):
        return not self.__eq__(other)

    def __hash__(self):
        return hash(self._name)

    def __repr__(self):
        return f"orca.{self._name}"


DType.FLOAT32 = DType("F32")
DType.FLOAT64 = DType("F64")
DType.FLOAT16 = DType("F16")
DType.BFLOAT16 = DType("BF16")
DType.INT32 = DType("I32")
DType.INT64 = DType("I64")
DType.UINT8 = DType("U8")
DType.BOOL = DType("Bool")


class Device:
    """orca.Device (orca-python/src/lib.rs:83-105); only "cpu" computes here."""

    def __init__(self, device_str: str):
        if device_str == "cpu":
            self.kind = "cpu"
        elif device_str.startswith("cuda") or device_str.startswith("gpu"):
            self.kind = "gpu"
        else:
            raise ValueError(f"Unknown device: {device_str}")

    def __repr__(self):
        return f"device(type='{self.kind}')"


def _check_device(device):
    if device is not None and isinstance(device, Device) and device.kind != "cpu":
        raise RuntimeError("the oracle stand-in only provides the CPU backend")


def _check_dtype(dtype):
    if dtype is not None and dtype != DType.FLOAT32:
        raise ValueError(f"UnsupportedDType: {dtype!r} (the oracle stand-in is FP32-only)")


# ---------------------------------------------------------------- tape
class _Tape:
    """orca-autograd/src/tape.rs:61-128: one global Wengert list."""

    def __init__(self):
        self.nodes = []
        self.next_id = 0
        self.grads = {}
        self.lock = threading.Lock()

    def generate_id(self):
        i = self.next_id
        self.next_id += 1
        return i

    def accumulate(self, node_id, g):
        if node_id in self.grads:
            self.grads[node_id] = O.accumulate_grad(self.grads[node_id], g).reshape(g.shape)
        else:
            self.grads[node_id] = g

    def clear(self):
        self.nodes.clear()
        self.grads.clear()


_TAPE = _Tape()
_GRAD = threading.local()


def set_grad_enabled(enabled: bool) -> None:
    _GRAD.enabled = bool(enabled)


def is_grad_enabled() -> bool:
    return getattr(_GRAD, "enabled", True)


def _record(node, *inputs):
    """Autodiff op wrapper pattern (orca-autograd/src/backend.rs:74-118): an id is
    generated whenever grad mode is on; a node is pushed only if an input
    requires grad."""
    if not is_grad_enabled():
        return None
    out_id = _TAPE.generate_id()
    if any(i is not None for i in inputs):
        node["out"] = out_id
        _TAPE.nodes.append(node)
        return out_id
    return None


def _backward_node(n):
    g = _TAPE.grads.get(n["out"])
    if g is None:
        return
    k = n["kind"]
    if k == "add":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], g)
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], g)
    elif k == "sub":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], g)
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], O.mul_scalar(g, -1.0))
    elif k == "mul_scalar":
        _TAPE.accumulate(n["in"], O.mul_scalar(g, n["s"]))
    elif k == "mul":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], O.mul(g, n["rp"]).reshape(g.shape))
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], O.mul(g, n["lp"]).reshape(g.shape))
    elif k == "div":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], O.div_backward_lhs(g, n["rp"]).reshape(g.shape))
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], O.div_backward_rhs(g, n["lp"], n["rp"]).reshape(g.shape))
    elif k == "matmul":
        ls, rs = n["ls"], n["rs"]
        r = len(ls)
        out_shape = list(ls)
        out_shape[r - 1] = rs[len(rs) - 1]
        if n["lhs"] is not None:
            rt = O.transpose(n["rp"], rs, len(rs) - 2, len(rs) - 1)
            _TAPE.accumulate(n["lhs"], O.matmul(g.reshape(out_shape), rt))
        if n["rhs"] is not None:
            lt = O.transpose(n["lp"], ls, r - 2, r - 1)
            _TAPE.accumulate(n["rhs"], O.matmul(lt, g.reshape(out_shape)))
    elif k == "transpose":
        oshape = list(n["shape"])
        oshape[n["d0"]], oshape[n["d1"]] = oshape[n["d1"]], oshape[n["d0"]]
        _TAPE.accumulate(n["in"], O.transpose(g, oshape, n["d0"], n["d1"]))
    elif k == "relu":
        _TAPE.accumulate(n["in"], O.relu_backward(g, n["ip"]).reshape(g.shape))
    elif k == "sigmoid":
        _TAPE.accumulate(n["in"], O.sigmoid_backward(g, n["op"]).reshape(g.shape))
    elif k == "sqrt":
        _TAPE.accumulate(n["in"], O.sqrt_backward(g, n["op"]).reshape(g.shape))
    elif k == "exp":
        _TAPE.accumulate(n["in"], O.exp_backward(g, n["op"]).reshape(g.shape))
    elif k == "log":
        _TAPE.accumulate(n["in"], O.log_backward(g, n["ip"]).reshape(g.shape))
    elif k == "expand":
        _TAPE.accumulate(n["in"], O.sum_to_shape(g, n["oshape"], n["ishape"]))
    elif k == "sum_to_shape":
        _TAPE.accumulate(n["in"], O.expand(g, n["oshape"], n["ishape"]))
    elif k == "reshape":
        _TAPE.accumulate(n["in"], g.reshape(n["ishape"]))
    elif k == "max_to_shape":
        gi = O.max_to_shape_backward(g, n["ip"], n["op"], n["ishape"], n["oshape"])
        _TAPE.accumulate(n["in"], gi)
    else:
        raise RuntimeError(f"unknown node {k}")


def _broadcast(a, b):
    """Shape::broadcast (orca-core/src/shape.rs:26-51)."""
    res = []
    i, j = len(a) - 1, len(b) - 1
    while i >= 0 or j >= 0:
        d1 = a[i] if i >= 0 else 1
        d2 = b[j] if j >= 0 else 1
        if d1 == d2:
            res.append(d1)
        elif d1 == 1:
            res.append(d2)
        elif d2 == 1:
            res.append(d1)
        else:
            return None
        i -= 1
        j -= 1
    return list(reversed(res))


# ---------------------------------------------------------------- tensor
class Tensor:
    """orca.Tensor over the restated CPU backend (orca-python/src/lib.rs:108-853)."""

    def __init__(self, data: np.ndarray, shape: List[int], node_id: Optional[int] = None):
        self._data = np.ascontiguousarray(data, dtype=np.float32).reshape(shape)
        self._shape = [int(s) for s in shape]
        self._node = node_id

    # -- factories
    @staticmethod
    def zeros(shape, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        _check_device(device)
        t = Tensor(np.zeros(int(np.prod(shape, dtype=np.int64)), np.float32), list(shape))
        if requires_grad:
            t.require_grad()
        return t

    @staticmethod
    def ones(shape, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        _check_device(device)
        t = Tensor(np.ones(int(np.prod(shape, dtype=np.int64)), np.float32), list(shape))
        if requires_grad:
            t.require_grad()
        return t

    @staticmethod
    def scalar(value, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        _check_device(device)
        t = Tensor(np.array([np.float32(value)]), [1])
        if requires_grad:
            t.require_grad()
        return t

    _rng = np.random.default_rng(12345)

    @staticmethod
    def rand_uniform(shape, low, high, dtype=None, device=None, requires_grad=False):
        # The reference draws from an unseeded thread_rng (orca-tensor/src/tensor.rs:63);
        # callers that need reproducibility overwrite the values, as the harness does.
        _check_dtype(dtype)
        n = int(np.prod(shape, dtype=np.int64))
        data = Tensor._rng.uniform(low, high, n).astype(np.float32)
        t = Tensor(data, list(shape))
        if requires_grad:
            t.require_grad()
        return t

    @staticmethod
    def randn(shape, mean=0.0, std=1.0, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        n = int(np.prod(shape, dtype=np.int64))
        t = Tensor(Tensor._rng.normal(mean, std, n).astype(np.float32), list(shape))
        if requires_grad:
            t.require_grad()
        return t

    @staticmethod
    def rand_dropout_mask(shape, p, dtype=None, device=None):
        n = int(np.prod(shape, dtype=np.int64))
        keep = (Tensor._rng.random(n) >= p).astype(np.float32)
        return Tensor(keep * np.float32(1.0 / (1.0 - p)), list(shape))

    @staticmethod
    def einsum(equation, inputs):
        raise ValueError("einsum is outside the MLP path of the oracle stand-in")

    @staticmethod
    def from_list(data, shape=None, requires_grad=False, device=None):
        _check_device(device)
        arr = np.asarray(data, dtype=np.float32).reshape(-1)
        shape = list(shape) if shape is not None else [arr.size]
        if int(np.prod(shape, dtype=np.int64)) != arr.size:
            raise ValueError("ShapeMismatch: data length does not match shape")
        t = Tensor(arr, shape)
        if requires_grad:
            t.require_grad()
        return t

    # -- properties
    def to(self, device_str):
        if device_str != "cpu":
            raise RuntimeError("the oracle stand-in only provides the CPU backend")
        return Tensor(self._data, self._shape, self._node)

    @property
    def shape(self):
        return list(self._shape)

    @property
    def dtype(self):
        return DType.FLOAT32

    @property
    def device(self):
        return Device("cpu")

    def to_list(self):
        return [float(v) for v in self._data.reshape(-1)]

    def numpy(self):
        """Stand-in convenience (not in the reference surface): a copy as ndarray."""
        return self._data.copy()

    # -- autograd ext (orca-autograd/src/tensor.rs)
    @property
    def requires_grad(self):
        return self._node is not None

    def require_grad(self):
        self._node = _TAPE.generate_id()

    def zero_grad(self):
        _TAPE.clear()

    def backward(self):
        if self._node is None:
            raise ValueError("Cannot call backward on a tensor that doesn't require gradients")
        _TAPE.grads[self._node] = np.ones(self._shape, np.float32)
        for n in reversed(_TAPE.nodes):
            _backward_node(n)

    def grad(self):
        if self._node is None:
            return None
        g = _TAPE.grads.get(self._node)
        if g is None:
            return None
        return Tensor(g, self._shape)

    def detach(self):
        return Tensor(self._data, self._shape, None)

    def set_grad(self, grad):
        if self._node is None:
            raise ValueError("tensor does not require grad")
        _TAPE.grads[self._node] = grad._data.reshape(self._shape).copy()

    def to_dtype(self, dtype):
        _check_dtype(dtype)
        return Tensor(self._data, self._shape, self._node)

    def has_nan_or_inf(self):
        return bool(not np.all(np.isfinite(self._data)))

    # -- shape ops
    def expand(self, shape):
        shape = list(shape)
        out = O.expand(self._data, self._shape, shape)
        nid = _record({"kind": "expand", "in": self._node, "ishape": self._shape,
                       "oshape": shape}, self._node)
        return Tensor(out, shape, nid)

    def sum_to_shape(self, shape):
        shape = list(shape)
        out = O.sum_to_shape(self._data, self._shape, shape)
        nid = _record({"kind": "sum_to_shape", "in": self._node, "ishape": self._shape,
                       "oshape": shape}, self._node)
        return Tensor(out, shape, nid)

    def max_to_shape(self, shape):
        shape = list(shape)
        out = O.max_to_shape(self._data, self._shape, shape)
        nid = _record({"kind": "max_to_shape", "in": self._node, "ishape": self._shape,
                       "oshape": shape, "ip": self._data, "op": out}, self._node)
        return Tensor(out, shape, nid)

    def reshape(self, shape):
        shape = list(shape)
        if int(np.prod(shape, dtype=np.int64)) != self._data.size:
            raise ValueError("ShapeMismatch: reshape element count")
        nid = _record({"kind": "reshape", "in": self._node, "ishape": self._shape,
                       "oshape": shape}, self._node)
        return Tensor(self._data, shape, nid)

    def transpose(self, dim0, dim1):
        out = O.transpose(self._data, self._shape, dim0, dim1)
        nid = _record({"kind": "transpose", "in": self._node, "shape": self._shape,
                       "d0": dim0, "d1": dim1}, self._node)
        return Tensor(out, list(out.shape), nid)

    def sum(self):
        return self.sum_to_shape([1])

    def mean(self):
        n = int(np.prod(self._shape, dtype=np.int64))
        return self.sum()._mul_scalar(np.float32(1.0) / np.float32(n))

    # -- elementwise
    def _same_shape(self, other, op):
        if self._shape != other._shape:
            raise ValueError(f"ShapeMismatch in {op}: {self._shape} vs {other._shape}")

    def _binary(self, other, kind, fn):
        self._same_shape(other, kind)
        out = fn(self._data, other._data).reshape(self._shape)
        node = {"kind": kind, "lhs": self._node, "rhs": other._node}
        if kind in ("mul", "div"):
            node["lp"], node["rp"] = self._data, other._data
        nid = _record(node, self._node, other._node)
        return Tensor(out, self._shape, nid)

    def _resolve(self, operand):
        if isinstance(operand, Tensor):
            return operand
        return Tensor.scalar(float(operand))

    def _bcast_pair(self, other):
        out_shape = _broadcast(self._shape, other._shape)
        if out_shape is None:
            raise ValueError("Shapes are not broadcastable")
        return self.expand(out_shape), other.expand(out_shape)

    def __add__(self, operand):
        s, o = self._bcast_pair(self._resolve(operand))
        return s._binary(o, "add", O.add)

    __radd__ = __add__

    def __sub__(self, operand):
        s, o = self._bcast_pair(self._resolve(operand))
        return s._binary(o, "sub", O.sub)

    def __rsub__(self, operand):
        other = self._resolve(operand)
        s, o = other._bcast_pair(self)
        return s._binary(o, "sub", O.sub)

    def _mul_scalar(self, s):
        s = np.float32(s)
        out = O.mul_scalar(self._data, s).reshape(self._shape)
        nid = _record({"kind": "mul_scalar", "in": self._node, "s": s}, self._node)
        return Tensor(out, self._shape, nid)

    def __mul__(self, operand):
        if not isinstance(operand, Tensor):
            return self._mul_scalar(np.float32(float(operand)))
        s, o = self._bcast_pair(operand)
        return s._binary(o, "mul", O.mul)

    __rmul__ = __mul__

    def __truediv__(self, operand):
        s, o = self._bcast_pair(self._resolve(operand))
        return s._binary(o, "div", O.div)

    def __rtruediv__(self, operand):
        other = self._resolve(operand)
        s, o = other._bcast_pair(self)
        return s._binary(o, "div", O.div)

    def __neg__(self):
        return self._mul_scalar(-1.0)

    def __matmul__(self, other):
        a, b = self._shape, other._shape
        if len(a) < 2 or len(b) < 2:
            raise ValueError("ShapeMismatch: matmul needs >= 2D tensors")
        if a[-1] != b[-2]:
            raise ValueError("ShapeMismatch: matmul inner dimensions")
        if len(a) != len(b) or a[:-2] != b[:-2]:
            raise ValueError("ShapeMismatch: matmul batch dimensions")
        out = O.matmul(self._data, other._data)
        nid = _record({"kind": "matmul", "lhs": self._node, "rhs": other._node,
                       "lp": self._data, "rp": other._data, "ls": a, "rs": b},
                      self._node, other._node)
        return Tensor(out, list(out.shape), nid)

    def _unary(self, kind, fn, keep):
        out = fn(self._data).reshape(self._shape)
        node = {"kind": kind, "in": self._node}
        if keep == "in":
            node["ip"] = self._data
        else:
            node["op"] = out
        nid = _record(node, self._node)
        return Tensor(out, self._shape, nid)

    def relu(self):
        return self._unary("relu", O.relu, "in")

    def sigmoid(self):
        return self._unary("sigmoid", O.sigmoid, "out")

    def sqrt(self):
        return self._unary("sqrt", O.sqrt, "out")

    def exp(self):
        return self._unary("exp", O.exp, "out")

    def log(self):
        return self._unary("log", O.log, "in")

    def __repr__(self):
        return f"Tensor(shape={self._shape}, dtype=F32, device=cpu)"


def save_tensors(path, tensors_dict):
    raise RuntimeError("serialization is outside the MLP path of the oracle stand-in")


def load_tensors(path):
    raise RuntimeError("serialization is outside the MLP path of the oracle stand-in")


def install(reference_python_dir: str):
    """Register this module as `orca.orca_python` and import the reference's
    pure-Python `orca` package from `reference_python_dir` on top of it."""
    import types

    mod = types.ModuleType("orca.orca_python")
    for name in ["Tensor", "DType", "Device", "save_tensors", "load_tensors",
                 "set_grad_enabled", "is_grad_enabled"]:
        setattr(mod, name, globals()[name])
    sys.modules["orca.orca_python"] = mod
    if reference_python_dir not in sys.path:
        sys.path.insert(0, reference_python_dir)
    import orca  # noqa: F401  (the reference package)
    return sys.modules["orca"]
