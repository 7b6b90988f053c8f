"""Python mirror of the reference's `Backend` trait on the CUDA library.

`CudaBackend` has one method per trait method the FP32 MLP path reaches
(orca-tensor/src/backend.rs:19-315), same names, same argument order and
meaning (storage handles + shapes + dtype), each returning a NEW storage the
way the trait does.  `CudaStorage` is the `Storage` (trait :7-15): a
refcounted device allocation, released when the Python object is collected.
Errors raise `OrcaError` (a ValueError, as PyO3 raises for OrcaError).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np

from . import _lib as L

F32, F64, F16, BF16, I32, I64, U8, BOOL = range(8)   # orca-core/src/dtype.rs:5-22
_NP = {F32: np.float32, F64: np.float64, F16: np.float16, I32: np.int32, I64: np.int64,
       U8: np.uint8, BOOL: np.bool_}


class CudaStorage:
    """A device buffer owned through the library's refcount."""

    __slots__ = ("_h", "backend")

    def __init__(self, handle, backend: "CudaBackend"):
        self._h = handle
        self.backend = backend

    def __len__(self):
        return int(L.load().orca_buf_len(self._h))

    @property
    def dtype(self) -> int:
        return int(L.load().orca_buf_dtype(self._h))

    @property
    def device_ptr(self) -> int:
        return int(L.load().orca_buf_device_ptr(self._h) or 0)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                L.load().orca_buf_release(h)
            except Exception:
                pass
            self._h = None


class CudaBackend:
    """One per device, like the reference's GpuBackend singleton
    (orca-python/src/lib.rs:23-33)."""

    def __init__(self, device: int = 0):
        lib = L.load()
        h = ctypes.c_void_p()
        L.check(lib.orca_ctx_create(int(device), ctypes.byref(h)))
        self._ctx = h
        self.device_index = int(device)

    def close(self):
        if getattr(self, "_ctx", None):
            L.load().orca_ctx_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def ctx(self):
        return self._ctx

    def device(self) -> str:
        return f"cuda:{self.device_index}"

    def synchronize(self, timeout_s: float = 600.0):
        L.check(L.load().orca_ctx_sync(self._ctx, float(timeout_s)))

    def set_timeout(self, seconds: float):
        """Deadline for every call that waits on the device; past it the call
        raises OrcaTimeout instead of blocking."""
        L.check(L.load().orca_ctx_set_timeout(self._ctx, float(seconds)))

    def selftest_wait_timeout(self, limit_s: float):
        """Runs a device wait that nothing completes, bounded by limit_s; raises
        OrcaTimeout (the expected outcome) and leaves the context usable."""
        L.check(L.load().orca_ctx_selftest_wait_timeout(self._ctx, float(limit_s)))

    def launch_count(self) -> int:
        return int(L.load().orca_ctx_launch_count(self._ctx))

    def stream_handle(self) -> int:
        return int(L.load().orca_ctx_stream(self._ctx) or 0)

    # -- helpers
    def _out(self, fn, *args) -> CudaStorage:
        out = ctypes.c_void_p()
        L.check(fn(self._ctx, *args, ctypes.byref(out)))
        return CudaStorage(out, self)

    # -- trait methods ---------------------------------------------------------
    def zeros(self, shape: Sequence[int], dtype: int = F32) -> CudaStorage:
        d, r = L.dims(shape)
        return self._out(L.load().orca_zeros, d, r, int(dtype))

    def from_f32_slice(self, shape: Sequence[int], data) -> CudaStorage:
        a = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        if a.size != int(np.prod(shape, dtype=np.int64)):
            raise L.OrcaError(1, "from_f32_slice: data length does not match shape")
        d, r = L.dims(shape)
        return self._out(L.load().orca_from_f32_slice, d, r, a.ctypes.data_as(ctypes.c_void_p))

    def to_f32_vec(self, storage: CudaStorage) -> np.ndarray:
        n = len(storage)
        out = np.empty(n, dtype=np.float32)
        L.check(L.load().orca_to_f32_vec(self._ctx, storage._h, out.ctypes.data_as(ctypes.c_void_p), n))
        return out

    def from_bytes(self, shape, data: bytes, dtype: int) -> CudaStorage:
        d, r = L.dims(shape)
        buf = ctypes.create_string_buffer(bytes(data), len(data))
        return self._out(L.load().orca_from_bytes, d, r, ctypes.cast(buf, ctypes.c_void_p),
                         len(data), int(dtype))

    def to_bytes(self, storage: CudaStorage) -> bytes:
        n = len(storage) * np.dtype(_NP.get(storage.dtype, np.uint16)).itemsize
        buf = ctypes.create_string_buffer(n)
        L.check(L.load().orca_to_bytes(self._ctx, storage._h, ctypes.cast(buf, ctypes.c_void_p), n))
        return buf.raw

    def matmul(self, lhs, rhs, lhs_shape, rhs_shape, dtype=F32) -> CudaStorage:
        dl, rl = L.dims(lhs_shape)
        dr, rr = L.dims(rhs_shape)
        return self._out(L.load().orca_matmul, lhs._h, rhs._h, dl, rl, dr, rr, int(dtype))

    def transpose(self, storage, shape, dim0, dim1, dtype=F32) -> CudaStorage:
        d, r = L.dims(shape)
        return self._out(L.load().orca_transpose, storage._h, d, r, int(dim0), int(dim1), int(dtype))

    def _bin(self, name, lhs, rhs, shape, dtype):
        d, r = L.dims(shape)
        return self._out(getattr(L.load(), "orca_" + name), lhs._h, rhs._h, d, r, int(dtype))

    def add(self, lhs, rhs, shape, dtype=F32): return self._bin("add", lhs, rhs, shape, dtype)
    def sub(self, lhs, rhs, shape, dtype=F32): return self._bin("sub", lhs, rhs, shape, dtype)
    def mul(self, lhs, rhs, shape, dtype=F32): return self._bin("mul", lhs, rhs, shape, dtype)
    def div(self, lhs, rhs, shape, dtype=F32): return self._bin("div", lhs, rhs, shape, dtype)

    def relu_backward(self, grad_out, in_primal, shape, dtype=F32):
        return self._bin("relu_backward", grad_out, in_primal, shape, dtype)

    def sigmoid_backward(self, grad_out, out_primal, shape, dtype=F32):
        return self._bin("sigmoid_backward", grad_out, out_primal, shape, dtype)

    def exp_backward(self, grad_out, out_primal, shape, dtype=F32):
        return self._bin("exp_backward", grad_out, out_primal, shape, dtype)

    def log_backward(self, grad_out, in_primal, shape, dtype=F32):
        return self._bin("log_backward", grad_out, in_primal, shape, dtype)

    def sqrt_backward(self, grad_out, out_primal, shape, dtype=F32):
        return self._bin("sqrt_backward", grad_out, out_primal, shape, dtype)

    def div_backward_lhs(self, grad_out, rhs_primal, shape, dtype=F32):
        return self._bin("div_backward_lhs", grad_out, rhs_primal, shape, dtype)

    def div_backward_rhs(self, grad_out, lhs_primal, rhs_primal, shape, dtype=F32):
        d, r = L.dims(shape)
        return self._out(L.load().orca_div_backward_rhs, grad_out._h, lhs_primal._h, rhs_primal._h,
                         d, r, int(dtype))

    def mul_scalar(self, storage, scalar, shape, dtype=F32):
        d, r = L.dims(shape)
        return self._out(L.load().orca_mul_scalar, storage._h, ctypes.c_float(np.float32(scalar)),
                         d, r, int(dtype))

    def _un(self, name, storage, shape, dtype):
        d, r = L.dims(shape)
        return self._out(getattr(L.load(), "orca_" + name), storage._h, d, r, int(dtype))

    def relu(self, s, shape, dtype=F32): return self._un("relu", s, shape, dtype)
    def sigmoid(self, s, shape, dtype=F32): return self._un("sigmoid", s, shape, dtype)
    def exp(self, s, shape, dtype=F32): return self._un("exp", s, shape, dtype)
    def log(self, s, shape, dtype=F32): return self._un("log", s, shape, dtype)
    def sqrt(self, s, shape, dtype=F32): return self._un("sqrt", s, shape, dtype)

    def _shape_op(self, name, storage, in_shape, out_shape, dtype):
        di, ri = L.dims(in_shape)
        do, ro = L.dims(out_shape)
        return self._out(getattr(L.load(), "orca_" + name), storage._h, di, ri, do, ro, int(dtype))

    def expand(self, s, in_shape, out_shape, dtype=F32):
        return self._shape_op("expand", s, in_shape, out_shape, dtype)

    def sum_to_shape(self, s, in_shape, out_shape, dtype=F32):
        return self._shape_op("sum_to_shape", s, in_shape, out_shape, dtype)

    def reshape(self, s, in_shape, out_shape, dtype=F32):
        return self._shape_op("reshape", s, in_shape, out_shape, dtype)

    def max_to_shape(self, s, in_shape, out_shape, dtype=F32):
        return self._shape_op("max_to_shape", s, in_shape, out_shape, dtype)

    def max_to_shape_backward(self, grad_out, in_primal, out_primal, in_shape, out_shape, dtype=F32):
        di, ri = L.dims(in_shape)
        do, ro = L.dims(out_shape)
        return self._out(L.load().orca_max_to_shape_backward, grad_out._h, in_primal._h,
                         out_primal._h, di, ri, do, ro, int(dtype))

    def accumulate_grad(self, lhs, rhs):
        return self._out(L.load().orca_accumulate_grad, lhs._h, rhs._h)

    def cast(self, storage, shape, current_dtype, target_dtype):
        d, r = L.dims(shape)
        return self._out(L.load().orca_cast, storage._h, d, r, int(current_dtype), int(target_dtype))

    def has_nan_or_inf(self, storage, dtype=F32) -> bool:
        res = ctypes.c_int()
        L.check(L.load().orca_has_nan_or_inf(self._ctx, storage._h, int(dtype), ctypes.byref(res)))
        return bool(res.value)

    # -- fused ops (inherent methods, not in the trait) ---------------------
    def linear_fwd(self, x, w, b, m, k, n, relu=False):
        return self._out(L.load().orca_linear_fwd, x._h, w._h, b._h if b is not None else None,
                         int(m), int(k), int(n), 1 if relu else 0)

    def linear_bwd(self, x, w, dy, m, k, n, mask=None, need_dx=True):
        """(dx or None, dw, db) of out = x @ w + b; dx masked by mask > 0."""
        dx, dw, db = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        L.check(L.load().orca_linear_bwd(self._ctx, x._h, w._h, dy._h,
                                         mask._h if mask is not None else None, int(m), int(k),
                                         int(n), ctypes.byref(dx) if need_dx else None,
                                         ctypes.byref(dw), ctypes.byref(db)))
        return (CudaStorage(dx, self) if need_dx else None, CudaStorage(dw, self),
                CudaStorage(db, self))

    def gemm_ex(self, m, n, k, a, a_mn_major, b, b_mn_major, path=0):
        return self._out(L.load().orca_gemm_ex, int(m), int(n), int(k), a._h,
                         1 if a_mn_major else 0, b._h, 1 if b_mn_major else 0, int(path))

    def softmax_ce_fwd_bwd(self, logits, target, batch, classes):
        loss = ctypes.c_void_p()
        dp = ctypes.c_void_p()
        L.check(L.load().orca_softmax_ce_fwd_bwd(self._ctx, logits._h, target._h, int(batch),
                                                 int(classes), ctypes.byref(loss), ctypes.byref(dp)))
        return CudaStorage(loss, self), CudaStorage(dp, self)

    def sgd_step(self, p, g, v, lr, momentum=0.0, dampening=0.0, weight_decay=0.0, first=False):
        L.check(L.load().orca_sgd_step(self._ctx, p._h, g._h, v._h if v is not None else None,
                                       lr, momentum, dampening, weight_decay, 1 if first else 0))

    def adamw_step(self, p, g, m, v, lr, beta1, beta2, eps, weight_decay, t):
        L.check(L.load().orca_adamw_step(self._ctx, p._h, g._h, m._h, v._h, lr, beta1, beta2, eps,
                                         weight_decay, int(t)))
