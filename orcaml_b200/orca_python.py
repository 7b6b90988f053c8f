"""A drop-in for the reference's compiled module `orca.orca_python`
(orca-python/src/lib.rs:909-919) on the CUDA library.

It exports the same names -- `Tensor`, `DType`, `Device`, `save_tensors`,
`load_tensors`, `set_grad_enabled`, `is_grad_enabled` -- with the same
arguments and errors, so the reference's pure-Python package (`orca.nn`,
`orca.optim`, `orca.distributed`, `Model.fit`) runs unchanged on a B200 once
`install()` has registered this module as `orca.orca_python`:

    import orcaml_b200.orca_python as op
    op.install()          # before `import orca`
    import orca           # the reference package, now on the GPU

Differences from the reference, all deliberate:
* Every tensor lives on the CUDA library (device index from `device`,
  "cpu" and None meaning device 0): the reference resolves "cuda" to its wgpu
  backend (lib.rs:91-93) and keeps "cpu" tensors on the host; here there is no
  host compute path at all.  `Tensor.device` reports the CUDA device and
  `Tensor.to(...)` moves between CUDA devices only.
* Operations run on the Backend-trait entry points of the C ABI
  (`CudaBackend`), each returning a new device buffer, as the trait does.
* Autograd is the reference's tape (orca-autograd/src/tape.rs:61-128): one
  global Wengert list, an id per result while grad mode is on, a node only
  when an input requires grad, reverse-order execution, gradients summed with
  `accumulate_grad`.  The backward rules are those of
  orca-autograd/src/backend.rs:1283-1930, expressed with the trait's own
  backward primitives (relu_backward, log_backward, ...).
* `einsum`, `conv2d`, `gather` and `scatter` are outside the FP32 MLP path and
  raise ValueError, as the library's NOT_IMPLEMENTED status does.
* `rand_uniform`/`randn`/`rand_dropout_mask` draw on the host (the reference
  uses an unseeded thread RNG, orca-tensor/src/tensor.rs:63,90) and upload.
"""
from __future__ import annotations

import sys
import threading
import types
from typing import Dict, List, Optional

import numpy as np

from . import safetensors_io
from .backend import BF16, BOOL, F16, F32, F64, I32, I64, U8, CudaBackend, CudaStorage

# ---------------------------------------------------------------- devices
_BACKENDS: Dict[int, CudaBackend] = {}
_BACKENDS_LOCK = threading.Lock()


def _backend(index: int = 0) -> CudaBackend:
    """One context per device, created on first use (lib.rs:18-33 keeps one
    backend singleton per kind)."""
    with _BACKENDS_LOCK:
        be = _BACKENDS.get(index)
        if be is None:
            try:
                be = CudaBackend(index)
            except Exception as exc:  # construction failures are RuntimeError (lib.rs:23-33)
                raise RuntimeError(f"Failed to initialise the CUDA backend on device {index}: "
                                   f"{exc}") from exc
            _BACKENDS[index] = be
        return be


class DType:
    """orca-python/src/lib.rs:41-80."""

    __slots__ = ("name", "code")

    def __init__(self, name: str, code: int):
        self.name = name
        self.code = code

    def __eq__(self, other):
        if not isinstance(other, DType):
            raise TypeError("Only Eq and Ne are supported between DTypes")
        return self.code == other.code

    def __ne__(self, other):
        return not self.__eq__(other)

    def __hash__(self):
        return hash(self.code)

    def __repr__(self):
        return f"orca.{self.name}"


DType.FLOAT32 = DType("F32", F32)
DType.FLOAT64 = DType("F64", F64)
DType.FLOAT16 = DType("F16", F16)
DType.BFLOAT16 = DType("BF16", BF16)
DType.INT32 = DType("I32", I32)
DType.INT64 = DType("I64", I64)
DType.UINT8 = DType("U8", U8)
DType.BOOL = DType("Bool", BOOL)
_DTYPES = {d.code: d for d in (DType.FLOAT32, DType.FLOAT64, DType.FLOAT16, DType.BFLOAT16,
                               DType.INT32, DType.INT64, DType.UINT8, DType.BOOL)}


class Device:
    """orca-python/src/lib.rs:82-104: "cpu", "cuda[:i]" or "gpu[:i]"."""

    __slots__ = ("kind", "index")

    def __init__(self, device_str: str):
        if device_str == "cpu":
            self.kind, self.index = "cpu", 0
        elif device_str.startswith("cuda") or device_str.startswith("gpu"):
            parts = device_str.split(":")
            try:
                self.index = int(parts[1]) if len(parts) > 1 else 0
            except ValueError:
                self.index = 0
            self.kind = "cuda"
        else:
            raise ValueError(f"Unknown device: {device_str}")

    def __repr__(self):
        return f"device(type='{self.kind}')" if self.kind == "cpu" else \
            f"device(type='cuda:{self.index}')"


def _device_index(device) -> int:
    if device is None:
        return 0
    if isinstance(device, Device):
        return device.index
    return Device(str(device)).index


def _check_dtype(dtype):
    if dtype is not None and dtype != DType.FLOAT32:
        raise ValueError("UnsupportedDType: the CUDA path computes in F32")


# ---------------------------------------------------------------- tape
class _Tape:
    """orca-autograd/src/tape.rs:61-128: one global Wengert list."""

    def __init__(self):
        self.nodes: list = []
        self.next_id = 0
        self.grads: dict = {}
        self.lock = threading.Lock()

    def generate_id(self) -> int:
        with self.lock:
            i = self.next_id
            self.next_id += 1
            return i

    def accumulate(self, node_id, g: "Tensor"):
        """Gradients::accumulate (tape.rs:34-47): sum with accumulate_grad."""
        prev = self.grads.get(node_id)
        if prev is None:
            self.grads[node_id] = g
        else:
            st = prev._be.accumulate_grad(prev._s, g._s)
            self.grads[node_id] = Tensor._wrap(st, prev._shape, prev._be)

    def clear(self):
        with self.lock:
            self.nodes.clear()
            self.grads.clear()


_TAPE = _Tape()
_GRAD = threading.local()


def set_grad_enabled(enabled: bool) -> None:
    """Thread-local grad mode (orca-autograd's GRAD_ENABLED, lib.rs:856-863)."""
    _GRAD.enabled = bool(enabled)


def is_grad_enabled() -> bool:
    return getattr(_GRAD, "enabled", True)


def _record(node: dict, *inputs) -> Optional[int]:
    """Autodiff op wrapper (orca-autograd/src/backend.rs:74-118): an id for
    every result while grad mode is on; a node only if an input needs grad."""
    if not is_grad_enabled():
        return None
    out_id = _TAPE.generate_id()
    if any(i is not None for i in inputs):
        node["out"] = out_id
        with _TAPE.lock:
            _TAPE.nodes.append(node)
        return out_id
    return None


def _backward_node(n: dict):
    g = _TAPE.grads.get(n["out"])
    if g is None:
        return
    be, k, gs = g._be, n["kind"], g._shape
    W = Tensor._wrap
    if k == "add":
        for side in ("lhs", "rhs"):
            if n[side] is not None:
                _TAPE.accumulate(n[side], g)
    elif k == "sub":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], g)
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], W(be.mul_scalar(g._s, -1.0, gs), gs, be))
    elif k == "mul_scalar":
        _TAPE.accumulate(n["in"], W(be.mul_scalar(g._s, n["s"], gs), gs, be))
    elif k == "mul":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], W(be.mul(g._s, n["rp"], gs), gs, be))
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], W(be.mul(g._s, n["lp"], gs), gs, be))
    elif k == "div":
        if n["lhs"] is not None:
            _TAPE.accumulate(n["lhs"], W(be.div_backward_lhs(g._s, n["rp"], gs), gs, be))
        if n["rhs"] is not None:
            _TAPE.accumulate(n["rhs"], W(be.div_backward_rhs(g._s, n["lp"], n["rp"], gs), gs, be))
    elif k == "matmul":
        # MatMulBackward (backend.rs:1448-1499): dA = g B^T, dB = A^T g.
        ls, rs = n["ls"], n["rs"]
        r = len(ls)
        if n["lhs"] is not None:
            rt_shape = rs[:-2] + [rs[-1], rs[-2]]
            rt = be.transpose(n["rp"], rs, r - 2, r - 1)
            _TAPE.accumulate(n["lhs"], W(be.matmul(g._s, rt, gs, rt_shape), ls, be))
        if n["rhs"] is not None:
            lt_shape = ls[:-2] + [ls[-1], ls[-2]]
            lt = be.transpose(n["lp"], ls, r - 2, r - 1)
            _TAPE.accumulate(n["rhs"], W(be.matmul(lt, g._s, lt_shape, gs), rs, be))
    elif k == "transpose":
        _TAPE.accumulate(n["in"], W(be.transpose(g._s, gs, n["d0"], n["d1"]), n["shape"], be))
    elif k == "relu":
        _TAPE.accumulate(n["in"], W(be.relu_backward(g._s, n["ip"], gs), gs, be))
    elif k == "sigmoid":
        _TAPE.accumulate(n["in"], W(be.sigmoid_backward(g._s, n["op"], gs), gs, be))
    elif k == "sqrt":
        _TAPE.accumulate(n["in"], W(be.sqrt_backward(g._s, n["op"], gs), gs, be))
    elif k == "exp":
        _TAPE.accumulate(n["in"], W(be.exp_backward(g._s, n["op"], gs), gs, be))
    elif k == "log":
        _TAPE.accumulate(n["in"], W(be.log_backward(g._s, n["ip"], gs), gs, be))
    elif k == "expand":
        _TAPE.accumulate(n["in"], W(be.sum_to_shape(g._s, n["oshape"], n["ishape"]),
                                    n["ishape"], be))
    elif k == "sum_to_shape":
        _TAPE.accumulate(n["in"], W(be.expand(g._s, n["oshape"], n["ishape"]), n["ishape"], be))
    elif k == "reshape":
        _TAPE.accumulate(n["in"], W(be.reshape(g._s, gs, n["ishape"]), n["ishape"], be))
    elif k == "max_to_shape":
        gi = be.max_to_shape_backward(g._s, n["ip"], n["op"], n["ishape"], n["oshape"])
        _TAPE.accumulate(n["in"], W(gi, n["ishape"], be))
    else:  # pragma: no cover - every recorded kind is handled above
        raise RuntimeError(f"unknown autograd node {k}")


def _broadcast(a: List[int], b: List[int]) -> Optional[List[int]]:
    """Shape::broadcast (orca-core/src/shape.rs:26-51)."""
    res = []
    i, j = len(a) - 1, len(b) - 1
    while i >= 0 or j >= 0:
        d1 = a[i] if i >= 0 else 1
        d2 = b[j] if j >= 0 else 1
        if d1 == d2 or d2 == 1:
            res.append(d1)
        elif d1 == 1:
            res.append(d2)
        else:
            return None
        i -= 1
        j -= 1
    return list(reversed(res))


def _numel(shape) -> int:
    return int(np.prod(shape, dtype=np.int64)) if len(shape) else 1


_RNG = np.random.default_rng()


# ---------------------------------------------------------------- tensor
class Tensor:
    """orca.Tensor (orca-python/src/lib.rs:106-853) on device memory."""

    __slots__ = ("_s", "_shape", "_node", "_be", "_dtype")

    def __init__(self, *args, **kwargs):
        raise TypeError("use Tensor.zeros/ones/scalar/from_list/... to create tensors")

    @classmethod
    def _wrap(cls, storage: CudaStorage, shape, be: CudaBackend, node=None, dtype: int = F32):
        t = object.__new__(cls)
        t._s = storage
        t._shape = [int(d) for d in shape]
        t._node = node
        t._be = be
        t._dtype = dtype
        return t

    @classmethod
    def _from_numpy(cls, arr: np.ndarray, shape, device=None, requires_grad=False):
        be = _backend(_device_index(device))
        t = cls._wrap(be.from_f32_slice(list(shape), np.ascontiguousarray(arr, np.float32)),
                      shape, be)
        if requires_grad:
            t.require_grad()
        return t

    # -- factories (lib.rs:155-421)
    @staticmethod
    def zeros(shape, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        be = _backend(_device_index(device))
        t = Tensor._wrap(be.zeros(list(shape)), list(shape), be)
        if requires_grad:
            t.require_grad()
        return t

    @staticmethod
    def ones(shape, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        return Tensor._from_numpy(np.ones(_numel(shape), np.float32), list(shape), device,
                                  requires_grad)

    @staticmethod
    def scalar(value, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        return Tensor._from_numpy(np.array([np.float32(value)]), [1], device, requires_grad)

    @staticmethod
    def rand_uniform(shape, low, high, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        data = _RNG.uniform(low, high, _numel(shape)).astype(np.float32)
        return Tensor._from_numpy(data, list(shape), device, requires_grad)

    @staticmethod
    def randn(shape, mean=0.0, std=1.0, dtype=None, device=None, requires_grad=False):
        _check_dtype(dtype)
        data = _RNG.normal(mean, std, _numel(shape)).astype(np.float32)
        return Tensor._from_numpy(data, list(shape), device, requires_grad)

    @staticmethod
    def rand_dropout_mask(shape, p, dtype=None, device=None):
        _check_dtype(dtype)
        if not (0.0 <= p < 1.0):
            raise ValueError("dropout probability must be in [0, 1)")
        keep = (_RNG.random(_numel(shape)) >= p).astype(np.float32)
        return Tensor._from_numpy(keep * np.float32(1.0 / (1.0 - p)), list(shape), device)

    @staticmethod
    def einsum(equation, inputs):
        raise ValueError("einsum is not implemented by the CUDA backend (not on the MLP path)")

    @staticmethod
    def from_list(data, shape=None, requires_grad=False, device=None):
        arr = np.asarray(data, dtype=np.float32).reshape(-1)
        shape = list(shape) if shape is not None else [arr.size]
        if _numel(shape) != arr.size:
            raise ValueError(f"Shape mismatch: data has {arr.size} elements, shape {shape}")
        return Tensor._from_numpy(arr, shape, device, requires_grad)

    # -- device / properties
    def to(self, device_str: str):
        idx = _device_index(device_str)
        if idx == self._be.device_index:
            return Tensor._wrap(self._s, self._shape, self._be, self._node, self._dtype)
        be = _backend(idx)
        st = be.from_bytes(self._shape, self._be.to_bytes(self._s), self._dtype)
        return Tensor._wrap(st, self._shape, be, self._node, self._dtype)

    @property
    def shape(self):
        return list(self._shape)

    @property
    def dtype(self):
        return _DTYPES[self._dtype]

    @property
    def device(self):
        return Device(f"cuda:{self._be.device_index}")

    def __repr__(self):
        return f"Tensor(shape={self._shape}, dtype={self.dtype!r}, device={self.device!r})"

    def to_list(self):
        if self._dtype != F32:
            return [float(v) for v in self._be.to_f32_vec(
                self._be.cast(self._s, self._shape, self._dtype, F32))]
        return [float(v) for v in self._be.to_f32_vec(self._s)]

    def numpy(self):
        """A host copy as ndarray (not in the reference surface; for tests)."""
        return self._be.to_f32_vec(self._s).reshape(self._shape)

    # -- autograd (orca-autograd/src/tensor.rs, lib.rs:787-853)
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
        _TAPE.grads[self._node] = Tensor.ones(self._shape, device=self.device)
        with _TAPE.lock:
            nodes = list(_TAPE.nodes)
        for n in reversed(nodes):
            _backward_node(n)

    def grad(self):
        if self._node is None:
            return None
        g = _TAPE.grads.get(self._node)
        return None if g is None else Tensor._wrap(g._s, self._shape, g._be)

    def detach(self):
        return Tensor._wrap(self._s, self._shape, self._be, None, self._dtype)

    def set_grad(self, grad: "Tensor"):
        if self._node is None:
            raise ValueError("Cannot set grad on a tensor that doesn't require gradients")
        if _numel(grad._shape) != _numel(self._shape):
            raise ValueError("Shape mismatch in set_grad")
        _TAPE.grads[self._node] = Tensor._wrap(grad._s, self._shape, grad._be)

    def to_dtype(self, dtype: DType):
        if dtype.code == self._dtype:
            return Tensor._wrap(self._s, self._shape, self._be, self._node, self._dtype)
        st = self._be.cast(self._s, self._shape, self._dtype, dtype.code)
        return Tensor._wrap(st, self._shape, self._be, None, dtype.code)

    def has_nan_or_inf(self) -> bool:
        return bool(self._be.has_nan_or_inf(self._s))

    # -- shape ops
    def expand(self, shape):
        shape = [int(d) for d in shape]
        st = self._be.expand(self._s, self._shape, shape)
        nid = _record({"kind": "expand", "in": self._node, "ishape": self._shape,
                       "oshape": shape}, self._node)
        return Tensor._wrap(st, shape, self._be, nid)

    def sum_to_shape(self, shape):
        shape = [int(d) for d in shape]
        st = self._be.sum_to_shape(self._s, self._shape, shape)
        nid = _record({"kind": "sum_to_shape", "in": self._node, "ishape": self._shape,
                       "oshape": shape}, self._node)
        return Tensor._wrap(st, shape, self._be, nid)

    def max_to_shape(self, shape):
        shape = [int(d) for d in shape]
        st = self._be.max_to_shape(self._s, self._shape, shape)
        nid = _record({"kind": "max_to_shape", "in": self._node, "ishape": self._shape,
                       "oshape": shape, "ip": self._s, "op": st}, self._node)
        return Tensor._wrap(st, shape, self._be, nid)

    def reshape(self, shape):
        shape = [int(d) for d in shape]
        if _numel(shape) != _numel(self._shape):
            raise ValueError(f"Shape mismatch: cannot reshape {self._shape} to {shape}")
        st = self._be.reshape(self._s, self._shape, shape)
        nid = _record({"kind": "reshape", "in": self._node, "ishape": self._shape}, self._node)
        return Tensor._wrap(st, shape, self._be, nid)

    def transpose(self, dim0: int, dim1: int):
        st = self._be.transpose(self._s, self._shape, dim0, dim1)
        out_shape = list(self._shape)
        out_shape[dim0], out_shape[dim1] = out_shape[dim1], out_shape[dim0]
        nid = _record({"kind": "transpose", "in": self._node, "shape": self._shape,
                       "d0": dim0, "d1": dim1}, self._node)
        return Tensor._wrap(st, out_shape, self._be, nid)

    def sum(self):
        return self.sum_to_shape([1])

    def mean(self):
        """sum * f32(1 / numel) (lib.rs:664-669)."""
        return self.sum()._mul_scalar(np.float32(1.0) / np.float32(_numel(self._shape)))

    # -- element-wise (lib.rs:495-660)
    def _check_peer(self, other: "Tensor"):
        if other._be is not self._be:
            raise ValueError("Cannot operate on tensors from different devices")

    def _binary(self, other: "Tensor", kind: str):
        self._check_peer(other)
        if self._shape != other._shape:
            raise ValueError(f"Shape mismatch in {kind}: {self._shape} vs {other._shape}")
        st = getattr(self._be, kind)(self._s, other._s, self._shape)
        node = {"kind": kind, "lhs": self._node, "rhs": other._node}
        if kind in ("mul", "div"):
            node["lp"], node["rp"] = self._s, other._s
        nid = _record(node, self._node, other._node)
        return Tensor._wrap(st, self._shape, self._be, nid)

    def _resolve(self, operand) -> "Tensor":
        if isinstance(operand, Tensor):
            return operand
        return Tensor.scalar(float(operand), device=self.device)

    def _bcast_pair(self, other: "Tensor"):
        out_shape = _broadcast(self._shape, other._shape)
        if out_shape is None:
            raise ValueError(f"Shapes {self._shape} and {other._shape} are not broadcastable")
        s = self if self._shape == out_shape else self.expand(out_shape)
        o = other if other._shape == out_shape else other.expand(out_shape)
        return s, o

    def __add__(self, operand):
        s, o = self._bcast_pair(self._resolve(operand))
        return s._binary(o, "add")

    def __radd__(self, operand):
        return self.__add__(operand)

    def __sub__(self, operand):
        s, o = self._bcast_pair(self._resolve(operand))
        return s._binary(o, "sub")

    def __rsub__(self, operand):
        s, o = self._resolve(operand)._bcast_pair(self)
        return s._binary(o, "sub")

    def _mul_scalar(self, s):
        s = float(np.float32(s))
        st = self._be.mul_scalar(self._s, s, self._shape)
        nid = _record({"kind": "mul_scalar", "in": self._node, "s": s}, self._node)
        return Tensor._wrap(st, self._shape, self._be, nid)

    def __mul__(self, operand):
        if not isinstance(operand, Tensor):
            return self._mul_scalar(np.float32(float(operand)))
        s, o = self._bcast_pair(operand)
        return s._binary(o, "mul")

    def __rmul__(self, operand):
        return self.__mul__(operand)

    def __truediv__(self, operand):
        s, o = self._bcast_pair(self._resolve(operand))
        return s._binary(o, "div")

    def __rtruediv__(self, operand):
        s, o = self._resolve(operand)._bcast_pair(self)
        return s._binary(o, "div")

    def __neg__(self):
        return self._mul_scalar(-1.0)

    def __matmul__(self, other: "Tensor"):
        self._check_peer(other)
        a, b = self._shape, other._shape
        if len(a) < 2 or len(b) < 2:
            raise ValueError("Shape mismatch: matmul needs tensors of rank >= 2")
        if a[-1] != b[-2] or len(a) != len(b) or a[:-2] != b[:-2]:
            raise ValueError(f"Shape mismatch in matmul: {a} @ {b}")
        st = self._be.matmul(self._s, other._s, a, b)
        out = a[:-1] + [b[-1]]
        nid = _record({"kind": "matmul", "lhs": self._node, "rhs": other._node,
                       "lp": self._s, "rp": other._s, "ls": list(a), "rs": list(b)},
                      self._node, other._node)
        return Tensor._wrap(st, out, self._be, nid)

    def _unary(self, kind: str, keep: str):
        st = getattr(self._be, kind)(self._s, self._shape)
        node = {"kind": kind, "in": self._node}
        node["ip" if keep == "in" else "op"] = self._s if keep == "in" else st
        nid = _record(node, self._node)
        return Tensor._wrap(st, self._shape, self._be, nid)

    def relu(self):
        return self._unary("relu", "in")

    def sigmoid(self):
        return self._unary("sigmoid", "out")

    def sqrt(self):
        return self._unary("sqrt", "out")

    def exp(self):
        return self._unary("exp", "out")

    def log(self):
        return self._unary("log", "in")

    def conv2d(self, weight, bias=None, padding=0, stride=1, dilation=1, groups=1):
        raise ValueError("conv2d is not implemented by the CUDA backend (not on the MLP path)")

    def gather(self, dim, index):
        raise ValueError("gather is not implemented by the CUDA backend (not on the MLP path)")

    def scatter(self, dim, index, src):
        raise ValueError("scatter is not implemented by the CUDA backend (not on the MLP path)")


# ---------------------------------------------------------------- safetensors
_ST_DTYPE = {F32: "F32", F64: "F64", F16: "F16", BF16: "BF16", I32: "I32", I64: "I64",
             U8: "U8", BOOL: "BOOL"}
_ST_CODE = {v: k for k, v in _ST_DTYPE.items()}


def save_tensors(path: str, tensors_dict: dict) -> None:
    """Writes the safetensors file orca-serialize writes
    (orca-serialize/src/lib.rs:6-38; layout in orcaml_b200.safetensors_io)."""
    if not isinstance(tensors_dict, dict):
        raise TypeError("tensors_dict must be a dict of name -> Tensor")
    entries = {}
    for name, t in tensors_dict.items():
        if not isinstance(t, Tensor):
            raise TypeError(f"{name!r} is not a Tensor")
        entries[str(name)] = (_ST_DTYPE[t._dtype], list(t._shape), t._be.to_bytes(t._s))
    try:
        safetensors_io.write(path, entries)
    except (OSError, ValueError) as exc:
        raise RuntimeError(f"Save failed: {exc}") from exc


def load_tensors(path: str, device=None) -> Dict[str, Tensor]:
    """Inverse of save_tensors (orca-serialize/src/lib.rs:40-79); every tensor
    is uploaded to the CUDA device (0 unless `device` says otherwise)."""
    try:
        entries, _ = safetensors_io.read(path)
    except (OSError, ValueError) as exc:
        raise RuntimeError(f"Load failed: {exc}") from exc
    be = _backend(_device_index(device))
    out = {}
    for name, (dtype, shape, data) in entries.items():
        code = _ST_CODE[dtype]
        out[name] = Tensor._wrap(be.from_bytes(shape, data, code), shape, be, None, code)
    return out


# ---------------------------------------------------------------- install
_EXPORTS = ["Tensor", "DType", "Device", "save_tensors", "load_tensors", "set_grad_enabled",
            "is_grad_enabled"]


def install() -> types.ModuleType:
    """Register this module as `orca.orca_python`, the name the reference's
    Python package imports its compiled core from; `import orca` afterwards
    runs the reference's pure-Python layers on the CUDA library."""
    mod = types.ModuleType("orca.orca_python")
    for name in _EXPORTS:
        setattr(mod, name, globals()[name])
    mod.__doc__ = __doc__
    sys.modules["orca.orca_python"] = mod
    return mod
