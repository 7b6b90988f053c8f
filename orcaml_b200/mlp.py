"""Device-resident training of Orca's Sequential(Linear, ReLU, ..., Linear) MLP.

`MlpTrainer` runs one step of

    optimizer.zero_grad(); loss = CrossEntropyLoss()(model(x), t); loss.backward();
    ddp.all_reduce_gradients(); optimizer.step()

(python/orca/nn/model.py:546-552, python/tests/test_phase8.py:119-126) as a
handful of fused CUDA kernels behind the C ABI (`orca_mlp_*`).  Parameters
follow Module.parameters() order (python/orca/nn/module.py:32-44): W0 [in,out],
b0 [1,out], W1, b1, ...; the optimizer hyper-parameters and their validation
follow python/orca/optim/sgd.py and adamw.py.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np

from . import _lib as L
from . import safetensors_io
from .backend import CudaBackend

OPT = {"sgd": 0, "adamw": 1}
GEMM_PATH = {"auto": 0, "simt": 1, "tc": 2, "tc_single": 3, "tc_pair": 4}


def _validate_float(name, value, positive=False):
    # python/orca/optim/optimizer.py:6-43
    if isinstance(value, bool):
        raise TypeError(f"{name} must be a finite float")
    try:
        v = float(value)
    except (TypeError, ValueError) as exc:
        raise TypeError(f"{name} must be a finite float") from exc
    if not np.isfinite(v):
        raise ValueError(f"{name} must be finite")
    if positive and v <= 0.0:
        raise ValueError(f"{name} must be positive")
    if not positive and v < 0.0:
        raise ValueError(f"{name} must be non-negative")
    return v


class MlpTrainer:
    def __init__(self, backend: CudaBackend, dims: Sequence[int], batch: int,
                 optimizer: str = "sgd", lr: float = 0.01, momentum: float = 0.0,
                 dampening: float = 0.0, weight_decay: float = 0.0,
                 betas=(0.9, 0.999), eps: float = 1e-8, gemm_path: str = "auto"):
        if optimizer not in OPT:
            raise ValueError(f"optimizer must be one of {sorted(OPT)}")
        lr = _validate_float("lr", lr)
        weight_decay = _validate_float("weight_decay", weight_decay)
        if optimizer == "sgd":
            momentum = _validate_float("momentum", momentum)
            dampening = _validate_float("dampening", dampening)
            if dampening > 1.0:
                raise ValueError("dampening must be in the range [0, 1]")
        else:
            try:
                b1, b2 = betas
            except (TypeError, ValueError) as exc:
                raise ValueError("betas must be a pair of floats") from exc
            for nm, b in (("betas[0]", b1), ("betas[1]", b2)):
                b = _validate_float(nm, b)
                if b >= 1.0:
                    raise ValueError(f"{nm} must be in the range [0, 1)")
            eps = _validate_float("eps", eps, positive=True)
        self.backend = backend
        self.dims = [int(d) for d in dims]
        self.batch = int(batch)
        self.optimizer = optimizer
        self._dims_arr = (ctypes.c_int64 * len(self.dims))(*self.dims)
        cfg = L.orca_mlp_config()
        cfg.n_layers = len(self.dims) - 1
        cfg.dims = ctypes.cast(self._dims_arr, L.P_int64)
        cfg.batch = self.batch
        cfg.optimizer = OPT[optimizer]
        cfg.lr, cfg.momentum, cfg.dampening, cfg.weight_decay = lr, momentum, dampening, weight_decay
        cfg.beta1, cfg.beta2 = float(betas[0]), float(betas[1])
        cfg.eps = float(eps)
        cfg.gemm_path = GEMM_PATH[gemm_path]
        h = ctypes.c_void_p()
        L.check(L.load().orca_mlp_create(backend.ctx, ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h
        self._comm = None

    # -- lifecycle
    def close(self):
        if getattr(self, "_h", None):
            L.load().orca_mlp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # -- parameters (Module.parameters() order)
    def param_shapes(self) -> List[tuple]:
        out = []
        for i in range(len(self.dims) - 1):
            out += [(self.dims[i], self.dims[i + 1]), (1, self.dims[i + 1])]
        return out

    def set_parameters(self, params: Sequence[np.ndarray]):
        shapes = self.param_shapes()
        if len(params) != len(shapes):
            raise ValueError(f"expected {len(shapes)} parameters, got {len(params)}")
        for i, (p, s) in enumerate(zip(params, shapes)):
            a = np.ascontiguousarray(p, dtype=np.float32)
            if a.size != s[0] * s[1]:
                raise ValueError(f"parameter {i}: expected shape {s}, got {a.shape}")
            L.check(L.load().orca_mlp_set_param(self._h, i, a.ctypes.data_as(ctypes.c_void_p), a.size))

    def get_parameters(self) -> List[np.ndarray]:
        out = []
        for i, s in enumerate(self.param_shapes()):
            a = np.empty(s, dtype=np.float32)
            L.check(L.load().orca_mlp_get_param(self._h, i, a.ctypes.data_as(ctypes.c_void_p), a.size))
            out.append(a)
        return out

    def get_grads(self) -> List[np.ndarray]:
        out = []
        for i, s in enumerate(self.param_shapes()):
            a = np.empty(s, dtype=np.float32)
            L.check(L.load().orca_mlp_get_grad(self._h, i, a.ctypes.data_as(ctypes.c_void_p), a.size))
            out.append(a)
        return out

    def get_activation(self, layer: int) -> np.ndarray:
        """Input of Linear `layer` (1..n_layers-1) in the last forward: the
        ReLU output of the layer below, [batch, dims[layer]]."""
        a = np.empty((self.batch, self.dims[layer]), dtype=np.float32)
        L.check(L.load().orca_mlp_get_activation(self._h, int(layer),
                                                 a.ctypes.data_as(ctypes.c_void_p), a.size))
        return a

    # -- checkpoints (safetensors)
    def param_names(self) -> List[str]:
        """The keys the reference's Module.save_weights gives the same model
        built as Sequential(Linear, ReLU, ..., Linear): modules are numbered in
        order (nn/container.py:10-11), the ReLUs take the odd indices, and
        Linear registers `weight` [in,out] and `bias` [1,out]
        (nn/module.py:169-187, nn/linear.py:29-36)."""
        out = []
        for i in range(len(self.dims) - 1):
            out += [f"{2 * i}.weight", f"{2 * i}.bias"]
        return out

    def save_weights(self, path: str):
        """Parameters only, in the file format and with the keys of the
        reference's Module.save_weights -- loadable by its load_weights."""
        entries = {n: ("F32", list(p.shape), p.tobytes())
                   for n, p in zip(self.param_names(), self.get_parameters())}
        safetensors_io.write(path, entries)

    def load_weights(self, path: str):
        """Reads a file written by save_weights or by the reference's
        Module.save_weights (keys and shapes must match this model)."""
        entries, _ = safetensors_io.read(path)
        params = []
        for name, shape in zip(self.param_names(), self.param_shapes()):
            if name not in entries:
                raise ValueError(f"{path}: missing tensor {name!r}")
            dtype, got, data = entries[name]
            if dtype != "F32" or int(np.prod(got)) != shape[0] * shape[1]:
                raise ValueError(f"{path}: {name!r} is {dtype} {got}, expected F32 {list(shape)}")
            params.append(np.frombuffer(data, np.float32).reshape(shape))
        self.set_parameters(params)

    def _state_slots(self):
        lib = L.load()
        slots = []
        for slot, suffix in ((0, "momentum_buffer" if self.optimizer == "sgd" else "exp_avg"),
                             (1, "exp_avg_sq")):
            n = ctypes.c_int64()
            L.check(lib.orca_mlp_state_numel(self._h, slot, 0, ctypes.byref(n)))
            if n.value:
                slots.append((slot, suffix))
        return slots

    def save_checkpoint(self, path: str):
        """Weights (as save_weights) plus the optimizer state the reference
        does not save: per parameter `optimizer.<key>.<slot>` tensors and the
        step counters in the file's metadata."""
        lib = L.load()
        entries = {n: ("F32", list(p.shape), p.tobytes())
                   for n, p in zip(self.param_names(), self.get_parameters())}
        for slot, suffix in self._state_slots():
            for i, (name, shape) in enumerate(zip(self.param_names(), self.param_shapes())):
                a = np.empty(shape, np.float32)
                L.check(lib.orca_mlp_get_state(self._h, slot, i, a.ctypes.data_as(ctypes.c_void_p),
                                               a.size))
                entries[f"optimizer.{name}.{suffix}"] = ("F32", list(shape), a.tobytes())
        t, started = ctypes.c_int64(), ctypes.c_int()
        L.check(lib.orca_mlp_get_step(self._h, ctypes.byref(t), ctypes.byref(started)))
        meta = {"format": "orcaml_b200.mlp", "optimizer": self.optimizer,
                "dims": ",".join(str(d) for d in self.dims), "step": str(t.value),
                "velocity_started": str(started.value)}
        safetensors_io.write(path, entries, meta)

    def load_checkpoint(self, path: str):
        """Restores weights, optimizer state and step counters written by
        save_checkpoint, so training continues bit-for-bit as if uninterrupted."""
        lib = L.load()
        entries, meta = safetensors_io.read(path)
        if meta.get("optimizer") != self.optimizer or \
                meta.get("dims") != ",".join(str(d) for d in self.dims):
            raise ValueError(f"{path}: checkpoint of a different model or optimizer")
        self.load_weights(path)
        for slot, suffix in self._state_slots():
            for i, (name, shape) in enumerate(zip(self.param_names(), self.param_shapes())):
                key = f"optimizer.{name}.{suffix}"
                if key not in entries:
                    raise ValueError(f"{path}: missing optimizer state {key!r}")
                a = np.ascontiguousarray(np.frombuffer(entries[key][2], np.float32))
                if a.size != shape[0] * shape[1]:
                    raise ValueError(f"{path}: {key!r} has the wrong size")
                L.check(lib.orca_mlp_set_state(self._h, slot, i, a.ctypes.data_as(ctypes.c_void_p),
                                               a.size))
        L.check(lib.orca_mlp_set_step(self._h, int(meta.get("step", "0")),
                                      int(meta.get("velocity_started", "0"))))

    # -- steps
    def _check_batch(self, x, t):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.shape != (self.batch, self.dims[0]):
            raise ValueError(f"x must be {(self.batch, self.dims[0])}, got {x.shape}")
        if t is not None:
            t = np.ascontiguousarray(t, dtype=np.float32)
            if t.shape != (self.batch, self.dims[-1]):
                raise ValueError(f"target must be {(self.batch, self.dims[-1])}, got {t.shape}")
        return x, t

    def step(self, x, t) -> float:
        """One training step from host arrays; returns this rank's loss."""
        x, t = self._check_batch(x, t)
        loss = ctypes.c_float()
        L.check(L.load().orca_mlp_step(self._h, x.ctypes.data_as(ctypes.c_void_p),
                                       t.ctypes.data_as(ctypes.c_void_p), ctypes.byref(loss)))
        return float(loss.value)

    def step_host_ptr(self, x_ptr: int, t_ptr: int, loss_host: Optional[ctypes.c_float] = None):
        """Step from raw host pointers (e.g. pinned buffers)."""
        L.check(L.load().orca_mlp_step(self._h, ctypes.c_void_p(x_ptr), ctypes.c_void_p(t_ptr),
                                       ctypes.byref(loss_host) if loss_host is not None else None))

    def step_device(self, x_dev: int, t_dev: int, loss_dev: int = 0):
        """Step from device pointers; enqueued only, nothing synchronised."""
        L.check(L.load().orca_mlp_step_device(self._h, ctypes.c_void_p(x_dev), ctypes.c_void_p(t_dev),
                                              ctypes.c_void_p(loss_dev) if loss_dev else None))

    def stage_batch(self, slot: int, x, t):
        """Copy a batch into device slot `slot` (0 or 1) on the step runner's
        copy stream.  With page-locked x and t (dataloader.pinned_empty) the
        call returns at once and the arrays must stay unchanged until the
        step on that slot has returned; pageable arrays are copied before it
        returns."""
        x, t = self._check_batch(x, t)
        L.check(L.load().orca_mlp_stage_batch(self._h, int(slot),
                                              x.ctypes.data_as(ctypes.c_void_p),
                                              t.ctypes.data_as(ctypes.c_void_p)))

    def step_staged(self, slot: int) -> float:
        """One training step on the batch staged in `slot`; returns the loss."""
        loss = ctypes.c_float()
        L.check(L.load().orca_mlp_step_staged(self._h, int(slot), ctypes.byref(loss)))
        return float(loss.value)

    def graph_capture(self, x_dev: int, t_dev: int, loss_dev: int = 0):
        """Record one step on fixed device buffers as a CUDA graph (SGD, no
        communicator); graph_step() then replays it with one launch."""
        L.check(L.load().orca_mlp_graph_capture(self._h, ctypes.c_void_p(x_dev),
                                                ctypes.c_void_p(t_dev),
                                                ctypes.c_void_p(loss_dev) if loss_dev else None))

    def graph_step(self):
        L.check(L.load().orca_mlp_graph_replay(self._h))

    def graph_release(self):
        L.check(L.load().orca_mlp_graph_release(self._h))

    def forward(self, x, t=None):
        """Logits [batch, classes] (and the loss when t is given)."""
        x, t = self._check_batch(x, t)
        logits = np.empty((self.batch, self.dims[-1]), np.float32)
        loss = ctypes.c_float(float("nan"))
        L.check(L.load().orca_mlp_forward(self._h, x.ctypes.data_as(ctypes.c_void_p),
                                          t.ctypes.data_as(ctypes.c_void_p) if t is not None else None,
                                          logits.ctypes.data_as(ctypes.c_void_p), ctypes.byref(loss)))
        return logits, (float(loss.value) if t is not None else None)

    def predict(self, x) -> np.ndarray:
        logits, _ = self.forward(x)
        return np.argmax(logits, axis=1)

    def launches_per_step(self) -> int:
        n = ctypes.c_int()
        L.check(L.load().orca_mlp_launches_per_step(self._h, ctypes.byref(n)))
        return int(n.value)

    def profile_begin(self):
        L.check(L.load().orca_mlp_profile_begin(self._h))

    def profile_end(self):
        """Per kernel group of the profiled steps: name, total ms, launches,
        FLOPs and bytes per launch, GEMM path (1 SIMT, 2 tcgen05, -1 other)."""
        lib = L.load()
        n = ctypes.c_int()
        L.check(lib.orca_mlp_profile_end(self._h, ctypes.byref(n)))
        out = []
        for i in range(n.value):
            name = ctypes.c_char_p()
            ms, fl, by = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
            cnt, path = ctypes.c_int(), ctypes.c_int()
            L.check(lib.orca_mlp_profile_site(self._h, i, ctypes.byref(name), ctypes.byref(ms),
                                              ctypes.byref(cnt), ctypes.byref(fl), ctypes.byref(by),
                                              ctypes.byref(path)))
            out.append({"name": name.value.decode(), "ms": ms.value, "launches": cnt.value,
                        "flops": fl.value, "bytes": by.value, "gemm_path": path.value})
        return out

    EXCHANGE = {"auto": 0, "nccl": 1, "peer": 2}

    def set_exchange(self, mode: str):
        """How gradients are averaged across ranks once a communicator is
        attached: "nccl" (ncclAllReduce, ncclAvg), "peer" (one kernel per
        layer over the ranks' IPC-mapped gradient arenas, float64 rank-order
        sum: the reference's average bit for bit) or "auto"."""
        if mode not in self.EXCHANGE:
            raise ValueError(f"exchange must be one of {sorted(self.EXCHANGE)}")
        L.check(L.load().orca_mlp_set_exchange(self._h, self.EXCHANGE[mode]))

    def exchange_kind(self) -> str:
        k = ctypes.c_int()
        L.check(L.load().orca_mlp_exchange_kind(self._h, ctypes.byref(k)))
        return {0: "none", 1: "nccl", 2: "peer"}[k.value]

    def attach_comm(self, comm, bucket_bytes: int = 0):
        self._comm = comm
        L.check(L.load().orca_mlp_attach_comm(self._h, comm.handle if comm is not None else None,
                                              int(bucket_bytes)))
