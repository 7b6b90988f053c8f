"""ctypes binding of liborca_cuda.so (the C ABI declared in include/orca_cuda.h).

The library is the product: there is no CPU or PyTorch fallback.  If the
shared object is missing this module raises at import time; build it with
`python -m orcaml_b200.build` (nvcc, sm_100a).
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liborca_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "orca_cuda.h")

c_int, c_int64, c_size_t, c_float, c_double = (ctypes.c_int, ctypes.c_int64, ctypes.c_size_t,
                                               ctypes.c_float, ctypes.c_double)
c_void_p, c_char_p, c_uint32, c_uint64 = (ctypes.c_void_p, ctypes.c_char_p, ctypes.c_uint32,
                                          ctypes.c_uint64)
P_int64 = ctypes.POINTER(c_int64)
P_float = ctypes.POINTER(c_float)
PP = ctypes.POINTER(c_void_p)

ORCA_OK = 0
STATUS_NAMES = {
    0: "ORCA_OK", 1: "ORCA_SHAPE_MISMATCH", 2: "ORCA_DEVICE_MISMATCH",
    3: "ORCA_UNSUPPORTED_DTYPE", 4: "ORCA_DTYPE_MISMATCH", 5: "ORCA_INTERNAL",
    6: "ORCA_TIMEOUT", 7: "ORCA_INVALID_ARGUMENT", 8: "ORCA_NOT_IMPLEMENTED",
    9: "ORCA_CUDA_ERROR", 10: "ORCA_COMM_ERROR",
}


class OrcaError(ValueError):
    """A failed call.  Subclasses ValueError because the reference's PyO3 layer
    maps every OrcaError to ValueError (orca-python/src/lib.rs:124)."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.status_name}: {message}")


class OrcaTimeout(OrcaError):
    pass


class OrcaCommError(OrcaError):
    pass


class orca_mlp_config(ctypes.Structure):
    _fields_ = [
        ("n_layers", c_int),
        ("dims", P_int64),
        ("batch", c_int64),
        ("optimizer", c_int),
        ("lr", c_double), ("momentum", c_double), ("dampening", c_double),
        ("weight_decay", c_double),
        ("beta1", c_double), ("beta2", c_double), ("eps", c_double),
        ("gemm_path", c_int),
    ]


# Argument types of every exported function (status-returning unless noted).
_SIGS = {
    "orca_last_error": ([], c_char_p),
    "orca_status_string": ([c_int], c_char_p),
    "orca_version": ([], c_uint32),
    "orca_ctx_create": ([c_int, PP], c_int),
    "orca_ctx_destroy": ([c_void_p], c_int),
    "orca_ctx_sync": ([c_void_p, c_double], c_int),
    "orca_ctx_device": ([c_void_p, ctypes.POINTER(c_int)], c_int),
    "orca_ctx_set_timeout": ([c_void_p, c_double], c_int),
    "orca_ctx_selftest_wait_timeout": ([c_void_p, c_double], c_int),
    "orca_ctx_stream": ([c_void_p], c_void_p),
    "orca_ctx_launch_count": ([c_void_p], c_uint64),
    "orca_buf_retain": ([c_void_p], c_int),
    "orca_buf_release": ([c_void_p], c_int),
    "orca_buf_len": ([c_void_p], c_size_t),
    "orca_buf_dtype": ([c_void_p], c_int),
    "orca_buf_device_ptr": ([c_void_p], c_void_p),
    "orca_zeros": ([c_void_p, P_int64, c_int, c_int, PP], c_int),
    "orca_from_f32_slice": ([c_void_p, P_int64, c_int, c_void_p, PP], c_int),
    "orca_to_f32_vec": ([c_void_p, c_void_p, c_void_p, c_size_t], c_int),
    "orca_from_bytes": ([c_void_p, P_int64, c_int, c_void_p, c_size_t, c_int, PP], c_int),
    "orca_to_bytes": ([c_void_p, c_void_p, c_void_p, c_size_t], c_int),
    "orca_matmul": ([c_void_p, c_void_p, c_void_p, P_int64, c_int, P_int64, c_int, c_int, PP], c_int),
    "orca_transpose": ([c_void_p, c_void_p, P_int64, c_int, c_int, c_int, c_int, PP], c_int),
    "orca_mul_scalar": ([c_void_p, c_void_p, c_float, P_int64, c_int, c_int, PP], c_int),
    "orca_accumulate_grad": ([c_void_p, c_void_p, c_void_p, PP], c_int),
    "orca_cast": ([c_void_p, c_void_p, P_int64, c_int, c_int, c_int, PP], c_int),
    "orca_has_nan_or_inf": ([c_void_p, c_void_p, c_int, ctypes.POINTER(c_int)], c_int),
    "orca_max_to_shape_backward": ([c_void_p, c_void_p, c_void_p, c_void_p, P_int64, c_int,
                                    P_int64, c_int, c_int, PP], c_int),
    "orca_div_backward_rhs": ([c_void_p, c_void_p, c_void_p, c_void_p, P_int64, c_int, c_int, PP],
                              c_int),
    "orca_conv2d": ([c_void_p, c_void_p, c_void_p, c_void_p, P_int64, c_int, P_int64, c_int,
                     c_int64, c_int64, c_int64, c_int64, c_int, PP], c_int),
    "orca_gather": ([c_void_p, c_void_p, c_int64, c_void_p, P_int64, c_int, P_int64, c_int, c_int,
                     PP], c_int),
    "orca_scatter": ([c_void_p, c_void_p, c_int64, c_void_p, c_void_p, P_int64, c_int, P_int64,
                      c_int, c_int, PP], c_int),
    "orca_mlp_graph_capture": ([c_void_p, c_void_p, c_void_p, c_void_p], c_int),
    "orca_mlp_graph_replay": ([c_void_p], c_int),
    "orca_mlp_graph_release": ([c_void_p], c_int),
    "orca_mlp_stage_batch": ([c_void_p, c_int, c_void_p, c_void_p], c_int),
    "orca_mlp_step_staged": ([c_void_p, c_int, c_void_p], c_int),
    "orca_host_alloc": ([c_size_t, PP], c_int),
    "orca_host_free": ([c_void_p], c_int),
    "orca_mlp_state_numel": ([c_void_p, c_int, c_int, P_int64], c_int),
    "orca_mlp_get_state": ([c_void_p, c_int, c_int, c_void_p, c_int64], c_int),
    "orca_mlp_set_state": ([c_void_p, c_int, c_int, c_void_p, c_int64], c_int),
    "orca_mlp_get_step": ([c_void_p, P_int64, ctypes.POINTER(c_int)], c_int),
    "orca_mlp_set_step": ([c_void_p, c_int64, c_int], c_int),
    "orca_linear_bwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                         c_int64, PP, PP, PP], c_int),
    "orca_linear_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                         PP], c_int),
    "orca_gemm_ex": ([c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_int, c_int,
                      PP], c_int),
    "orca_softmax_ce_fwd_bwd": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, PP, PP], c_int),
    "orca_softmax_ce_fwd_bwd_noalloc": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                         c_void_p], c_int),
    "orca_sgd_step": ([c_void_p, c_void_p, c_void_p, c_void_p, c_double, c_double, c_double,
                       c_double, c_int], c_int),
    "orca_adamw_step": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_double, c_double,
                         c_double, c_double, c_double, c_int64], c_int),
    "orca_mlp_create": ([c_void_p, ctypes.POINTER(orca_mlp_config), PP], c_int),
    "orca_mlp_destroy": ([c_void_p], c_int),
    "orca_mlp_num_params": ([c_void_p, ctypes.POINTER(c_int)], c_int),
    "orca_mlp_param_numel": ([c_void_p, c_int, P_int64], c_int),
    "orca_mlp_set_param": ([c_void_p, c_int, c_void_p, c_int64], c_int),
    "orca_mlp_get_param": ([c_void_p, c_int, c_void_p, c_int64], c_int),
    "orca_mlp_get_grad": ([c_void_p, c_int, c_void_p, c_int64], c_int),
    "orca_mlp_get_activation": ([c_void_p, c_int, c_void_p, c_int64], c_int),
    "orca_mlp_attach_comm": ([c_void_p, c_void_p, c_size_t], c_int),
    "orca_mlp_set_exchange": ([c_void_p, c_int], c_int),
    "orca_mlp_exchange_kind": ([c_void_p, ctypes.POINTER(c_int)], c_int),
    "orca_mlp_bucket_plan": ([c_int, P_int64, c_size_t, c_int, P_int64, P_int64,
                              ctypes.POINTER(c_int), ctypes.POINTER(c_int)], c_int),
    "orca_mlp_step": ([c_void_p, c_void_p, c_void_p, c_void_p], c_int),
    "orca_mlp_step_device": ([c_void_p, c_void_p, c_void_p, c_void_p], c_int),
    "orca_mlp_forward": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p], c_int),
    "orca_mlp_launches_per_step": ([c_void_p, ctypes.POINTER(c_int)], c_int),
    "orca_mlp_profile_begin": ([c_void_p], c_int),
    "orca_mlp_profile_end": ([c_void_p, ctypes.POINTER(c_int)], c_int),
    "orca_mlp_profile_site": ([c_void_p, c_int, ctypes.POINTER(c_char_p), ctypes.POINTER(c_double),
                               ctypes.POINTER(c_int), ctypes.POINTER(c_double),
                               ctypes.POINTER(c_double), ctypes.POINTER(c_int)], c_int),
    "orca_comm_get_unique_id": ([c_void_p], c_int),
    "orca_comm_init": ([c_void_p, c_int, c_int, c_void_p, c_double, PP], c_int),
    "orca_comm_destroy": ([c_void_p], c_int),
    "orca_comm_abort": ([c_void_p], c_int),
    "orca_comm_allreduce_avg": ([c_void_p, c_void_p, c_size_t], c_int),
    "orca_comm_allreduce_avg_bufs": ([c_void_p, PP, c_int, c_size_t], c_int),
}
# Element-wise binaries: (ctx, lhs, rhs, dims, rank, dtype, out)
for _n in ["add", "sub", "mul", "div", "relu_backward", "sigmoid_backward", "exp_backward",
           "log_backward", "sqrt_backward", "div_backward_lhs"]:
    _SIGS["orca_" + _n] = ([c_void_p, c_void_p, c_void_p, P_int64, c_int, c_int, PP], c_int)
# Element-wise unaries: (ctx, x, dims, rank, dtype, out)
for _n in ["relu", "sigmoid", "exp", "log", "sqrt"]:
    _SIGS["orca_" + _n] = ([c_void_p, c_void_p, P_int64, c_int, c_int, PP], c_int)
# Shape ops: (ctx, x, in_dims, in_rank, out_dims, out_rank, dtype, out)
for _n in ["expand", "sum_to_shape", "reshape", "max_to_shape"]:
    _SIGS["orca_" + _n] = ([c_void_p, c_void_p, P_int64, c_int, P_int64, c_int, c_int, PP], c_int)

_lib = None


def header_symbols():
    """Function names declared in include/orca_cuda.h."""
    with open(HEADER) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(orca_[a-z0-9_]+)\s*\(", text)))


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m orcaml_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in _SIGS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    _lib = lib
    return lib


def check(status: int):
    if status == ORCA_OK:
        return
    msg = load().orca_last_error().decode(errors="replace")
    if status == 6:
        raise OrcaTimeout(status, msg)
    if status == 10:
        raise OrcaCommError(status, msg)
    raise OrcaError(status, msg)


def dims(shape):
    shape = [int(s) for s in shape]
    arr = (c_int64 * max(1, len(shape)))(*shape)
    return arr, len(shape)
