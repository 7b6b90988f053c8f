"""numpy front end of the CPU oracle (liborca_oracle.so).

TEST INFRASTRUCTURE ONLY: this is the checker the CUDA backend is compared
against.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
arm import it; the product package (orcaml_b200) never does.

Every function wraps one C function of oracle/orca_oracle.c, which restates
the reference's CPU backend (orca-backend-cpu/src/backend.rs) and the
composition the reference's Python frontend + tape autograd perform for one
MLP training step (python/orca/nn, python/orca/optim, python/orca/distributed.py,
orca-autograd/src/backend.rs).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liborca_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)


def build(force: bool = False) -> str:
    """Compile liborca_oracle.so with oracle/Makefile (gcc, no GPU needed)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "orca_oracle.c"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    ew2 = ["oc_add", "oc_sub", "oc_mul", "oc_div", "oc_relu_backward", "oc_sigmoid_backward",
           "oc_exp_backward", "oc_log_backward", "oc_sqrt_backward", "oc_div_backward_lhs",
           "oc_accumulate_grad"]
    for name in ew2:
        f = getattr(L, name)
        f.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64]
        f.restype = None
    for name in ["oc_relu", "oc_sigmoid", "oc_exp", "oc_log", "oc_sqrt"]:
        f = getattr(L, name)
        f.argtypes = [_f32p, _f32p, ctypes.c_int64]
        f.restype = None
    L.oc_mul_scalar.argtypes = [_f32p, ctypes.c_float, _f32p, ctypes.c_int64]
    L.oc_div_backward_rhs.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int64]
    for name in ["oc_expand", "oc_sum_to_shape", "oc_max_to_shape"]:
        f = getattr(L, name)
        f.argtypes = [_f32p, _i64p, ctypes.c_int, _f32p, _i64p, ctypes.c_int]
        f.restype = ctypes.c_int
    L.oc_max_to_shape_backward.argtypes = [_f32p, _f32p, _f32p, _i64p, ctypes.c_int, _i64p,
                                           ctypes.c_int, _f32p]
    L.oc_max_to_shape_backward.restype = ctypes.c_int
    L.oc_transpose.argtypes = [_f32p, _i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
    L.oc_transpose.restype = ctypes.c_int
    L.oc_matmul.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                            ctypes.c_int64]
    PP = ctypes.POINTER(_f32p)
    L.oc_mlp_forward_backward.argtypes = [ctypes.c_int, _i64p, ctypes.c_int64, PP, PP, _f32p, _f32p,
                                          _f32p, PP, PP, _f32p]
    L.oc_mlp_forward_backward.restype = ctypes.c_int
    L.oc_mlp_forward.argtypes = [ctypes.c_int, _i64p, ctypes.c_int64, PP, PP, _f32p, _f32p, _f32p,
                                 _f32p]
    L.oc_mlp_forward.restype = ctypes.c_int
    L.oc_softmax_ce.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64, _f32p, _f32p]
    L.oc_sgd_step.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_double, ctypes.c_double,
                              ctypes.c_double, ctypes.c_double, ctypes.c_int]
    L.oc_adamw_step.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_double,
                                ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                ctypes.c_int64]
    L.oc_ddp_average.argtypes = [PP, ctypes.c_int, ctypes.c_int64, _f32p]
    L.oc_set_gemm_order.argtypes = [ctypes.c_int]
    L.oc_set_gemm_threads.argtypes = [ctypes.c_int]
    L.oc_sgemm_packed.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int64]
    L.oc_sgemm_packed.restype = ctypes.c_int
    L.oc_set_threads.argtypes = [ctypes.c_int]
    L.oc_get_threads.restype = ctypes.c_int


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _shape(s: Sequence[int]):
    arr = (ctypes.c_int64 * max(1, len(s)))(*[int(v) for v in s])
    return arr, len(s)


def set_threads(n: int) -> None:
    lib().oc_set_threads(int(n))


def set_gemm_order(order: int) -> None:
    """0: k ascending (default); 1: with FMA; 2: k-blocks of 256; 3: f64-rounded;
    4: the packed FMA kernel (timing stand-in for the reference's matrixmultiply)."""
    lib().oc_set_gemm_order(int(order))


def set_gemm_threads(n: int) -> None:
    """Threads of the default-order GEMM (1 = single-threaded like the
    reference; <= 0 = all).  Results are bit-identical at any count."""
    lib().oc_set_gemm_threads(int(n))


def sgemm_packed(a, b):
    """C = A @ B with the timing stand-in GEMM (None without AVX2/FMA)."""
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), np.float32)
    if lib().oc_sgemm_packed(_p(a), _p(b), _p(out), m, k, n) != 0:
        return None
    return out


def threads() -> int:
    return int(lib().oc_get_threads())


# ---- primitives -------------------------------------------------------------------
def _ew2(name):
    def f(a, b):
        a, b = _f32(a), _f32(b)
        assert a.size == b.size
        out = np.empty_like(a)
        getattr(lib(), name)(_p(a), _p(b), _p(out), a.size)
        return out
    f.__name__ = name[3:]
    return f


add = _ew2("oc_add")
sub = _ew2("oc_sub")
mul = _ew2("oc_mul")
div = _ew2("oc_div")
relu_backward = _ew2("oc_relu_backward")
sigmoid_backward = _ew2("oc_sigmoid_backward")
exp_backward = _ew2("oc_exp_backward")
log_backward = _ew2("oc_log_backward")
sqrt_backward = _ew2("oc_sqrt_backward")
div_backward_lhs = _ew2("oc_div_backward_lhs")
accumulate_grad = _ew2("oc_accumulate_grad")


def _ew1(name):
    def f(a):
        a = _f32(a)
        out = np.empty_like(a)
        getattr(lib(), name)(_p(a), _p(out), a.size)
        return out
    f.__name__ = name[3:]
    return f


relu = _ew1("oc_relu")
sigmoid = _ew1("oc_sigmoid")
exp = _ew1("oc_exp")
log = _ew1("oc_log")
sqrt = _ew1("oc_sqrt")


def mul_scalar(a, s: float):
    a = _f32(a)
    out = np.empty_like(a)
    lib().oc_mul_scalar(_p(a), ctypes.c_float(np.float32(s)), _p(out), a.size)
    return out


def div_backward_rhs(g, l, r):
    g, l, r = _f32(g), _f32(l), _f32(r)
    out = np.empty_like(g)
    lib().oc_div_backward_rhs(_p(g), _p(l), _p(r), _p(out), g.size)
    return out


def _shape_op(name):
    def f(a, in_shape, out_shape):
        a = _f32(a)
        si, ri = _shape(in_shape)
        so, ro = _shape(out_shape)
        out = np.empty(int(np.prod(out_shape, dtype=np.int64)), dtype=np.float32)
        rc = getattr(lib(), name)(_p(a), si, ri, _p(out), so, ro)
        if rc != 0:
            raise ValueError(f"{name}: bad shapes {in_shape} -> {out_shape}")
        return out.reshape(out_shape)
    f.__name__ = name[3:]
    return f


expand = _shape_op("oc_expand")
sum_to_shape = _shape_op("oc_sum_to_shape")
max_to_shape = _shape_op("oc_max_to_shape")


def max_to_shape_backward(g, in_primal, out_primal, in_shape, out_shape):
    g, ip, op = _f32(g), _f32(in_primal), _f32(out_primal)
    si, ri = _shape(in_shape)
    so, ro = _shape(out_shape)
    out = np.empty(int(np.prod(in_shape, dtype=np.int64)), dtype=np.float32)
    rc = lib().oc_max_to_shape_backward(_p(g), _p(ip), _p(op), si, ri, so, ro, _p(out))
    if rc != 0:
        raise ValueError("max_to_shape_backward: bad shapes")
    return out.reshape(in_shape)


def transpose(a, shape, dim0, dim1):
    a = _f32(a)
    s, r = _shape(shape)
    out = np.empty(a.size, dtype=np.float32)
    rc = lib().oc_transpose(_p(a), s, r, int(dim0), int(dim1), _p(out))
    if rc != 0:
        raise ValueError("transpose: bad dims")
    oshape = list(shape)
    oshape[dim0], oshape[dim1] = oshape[dim1], oshape[dim0]
    return out.reshape(oshape)


def matmul(a, b):
    """Batched row-major matmul with the reference's shape rules (same rank)."""
    a, b = _f32(a), _f32(b)
    assert a.ndim == b.ndim >= 2 and a.shape[:-2] == b.shape[:-2] and a.shape[-1] == b.shape[-2]
    m, k, n = a.shape[-2], a.shape[-1], b.shape[-1]
    batch = int(np.prod(a.shape[:-2], dtype=np.int64)) if a.ndim > 2 else 1
    out = np.empty(a.shape[:-2] + (m, n), dtype=np.float32)
    lib().oc_matmul(_p(a), _p(b), _p(out), batch, m, k, n)
    return out


# ---- composed step ---------------------------------------------------------------
def _ptr_array(arrs):
    return (_f32p * len(arrs))(*[_p(a) for a in arrs])


def mlp_forward_backward(dims: Sequence[int], params: List[np.ndarray], x, t
                         ) -> Tuple[float, List[np.ndarray], np.ndarray]:
    """One forward + CE + backward; params/grads in Module.parameters() order."""
    L = len(dims) - 1
    Ws = [_f32(params[2 * l]) for l in range(L)]
    bs = [_f32(params[2 * l + 1]) for l in range(L)]
    x, t = _f32(x), _f32(t)
    B = x.shape[0]
    dW = [np.empty((dims[l], dims[l + 1]), np.float32) for l in range(L)]
    db = [np.empty((1, dims[l + 1]), np.float32) for l in range(L)]
    logits = np.empty((B, dims[-1]), np.float32)
    loss = np.zeros(1, np.float32)
    d, _ = _shape(dims)
    rc = lib().oc_mlp_forward_backward(L, d, B, _ptr_array(Ws), _ptr_array(bs), _p(x), _p(t),
                                       _p(loss), _ptr_array(dW), _ptr_array(db), _p(logits))
    if rc != 0:
        raise ValueError("oc_mlp_forward_backward failed")
    grads = []
    for l in range(L):
        grads += [dW[l], db[l]]
    return float(loss[0]), grads, logits


def mlp_forward(dims, params, x, t):
    L = len(dims) - 1
    Ws = [_f32(params[2 * l]) for l in range(L)]
    bs = [_f32(params[2 * l + 1]) for l in range(L)]
    x, t = _f32(x), _f32(t)
    B = x.shape[0]
    logits = np.empty((B, dims[-1]), np.float32)
    loss = np.zeros(1, np.float32)
    d, _ = _shape(dims)
    rc = lib().oc_mlp_forward(L, d, B, _ptr_array(Ws), _ptr_array(bs), _p(x), _p(t), _p(loss),
                              _p(logits))
    if rc != 0:
        raise ValueError("oc_mlp_forward failed")
    return float(loss[0]), logits


def softmax_ce(P, T, with_grad=True):
    P, T = _f32(P), _f32(T)
    B, C = P.shape
    loss = np.zeros(1, np.float32)
    dP = np.empty_like(P) if with_grad else None
    lib().oc_softmax_ce(_p(P), _p(T), B, C, _p(loss), _p(dP) if with_grad else None)
    return float(loss[0]), dP


def sgd_step(p, g, v, lr, momentum=0.0, dampening=0.0, weight_decay=0.0, first=False):
    """In-place on p (and v)."""
    vp = _p(v) if v is not None else None
    lib().oc_sgd_step(_p(p), _p(_f32(g)), vp, p.size, lr, momentum, dampening, weight_decay,
                      1 if first else 0)


def adamw_step(p, g, m, v, lr, beta1, beta2, eps, weight_decay, t):
    lib().oc_adamw_step(_p(p), _p(_f32(g)), _p(m), _p(v), p.size, lr, beta1, beta2, eps,
                        weight_decay, int(t))


def ddp_average(rank_grads: List[np.ndarray]) -> np.ndarray:
    gs = [_f32(g) for g in rank_grads]
    out = np.empty_like(gs[0])
    lib().oc_ddp_average(_ptr_array(gs), len(gs), gs[0].size, _p(out))
    return out


class OracleTrainer:
    """Restated training loop: Sequential(Linear, ReLU, ..., Linear) +
    CrossEntropyLoss + SGD/AdamW (+ DDP averaging across rank inputs), the way
    python/orca/nn/model.py:546-552 and python/tests/test_phase8.py:119-126
    drive one step: zero_grad; forward; loss; backward; all_reduce; step."""

    def __init__(self, dims, params, optimizer="sgd", lr=0.01, momentum=0.0, dampening=0.0,
                 weight_decay=0.0, betas=(0.9, 0.999), eps=1e-8):
        self.dims = list(dims)
        self.params = [np.array(p, dtype=np.float32, copy=True) for p in params]
        self.opt = optimizer
        self.lr, self.momentum, self.dampening = lr, momentum, dampening
        self.weight_decay, self.betas, self.eps = weight_decay, betas, eps
        self.t = 0
        self.vel = [None] * len(self.params)
        if optimizer == "adamw":
            self.m = [np.zeros_like(p) for p in self.params]
            self.v = [np.zeros_like(p) for p in self.params]

    def grads(self, x, t):
        return mlp_forward_backward(self.dims, self.params, x, t)

    def apply(self, grads):
        if self.opt == "sgd":
            for i, (p, g) in enumerate(zip(self.params, grads)):
                first = False
                if self.momentum != 0.0 and self.vel[i] is None:
                    self.vel[i] = np.zeros_like(p)
                    first = True
                sgd_step(p, g, self.vel[i], self.lr, self.momentum, self.dampening,
                         self.weight_decay, first)
        elif self.opt == "adamw":
            self.t += 1
            for i, (p, g) in enumerate(zip(self.params, grads)):
                adamw_step(p, g, self.m[i], self.v[i], self.lr, self.betas[0], self.betas[1],
                           self.eps, self.weight_decay, self.t)
        else:
            raise ValueError(self.opt)

    def step(self, x, t):
        loss, grads, _ = self.grads(x, t)
        self.apply(grads)
        return loss

    def step_ddp(self, xs, ts):
        """All ranks' batches in one process; identical replicas by construction."""
        per = [self.grads(x, t) for x, t in zip(xs, ts)]
        avg = [ddp_average([p[1][i] for p in per]) for i in range(len(self.params))]
        self.apply(avg)
        return [p[0] for p in per]
