"""Benchmark: train samples/s of MLP 784-8192-8192-10 FP32 data-parallel
training (SGD momentum 0.9, lr 0.01, per-rank batch
4096) on N B200s, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c0|c1|c4]

The default workload is configs[2], the configuration BASELINE's metric is
quoted on; `--config` runs the other MLP configs the same way (their own
optimizer, inputs and shapes) for reference measurements.

A step is one full training step (forward, softmax-CE, backward, the
gradient exchange when N > 1 -- the peer-memory kernel by default, NCCL with
ORCA_XCHG=nccl -- and the optimizer update).  Every rank holds a
full replica and its own batch (weak scaling); `value` counts samples of all
ranks.  Timing: W untimed steps, then K steps bracketed by a barrier and a
device synchronise on both sides, timed with CUDA events on the library's
compute stream, max over ranks.  The step's working set (the 8192x8192
weight planes alone are 512 MB) exceeds the 126 MB L2, so no flush is needed.

At N > 1 every rank first runs a data-parallel parity pre-check outside the
timed region (`ddp_parity` in the JSON line; `--no-parity` skips it): a
reduced model through the same trainer, communicator and exchange, against
the oracle's restatement of the reference's DDP average.

`--impl reference` times the reference's CPU path restated in oracle/ (the
Rust reference cannot be built here) on the host cores, rank 0 only, with a
packed FMA GEMM standing in for the reference's matrixmultiply crate; steps
are timed on 128- and 512-row samples and `value` is their fixed + per-row
fit at the configuration's batch.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from orcaml_b200.synthetic import CONFIGS, init_params, make_batch  # noqa: E402

CFG = CONFIGS["c2"]
METRIC_C2 = "train samples/s, MLP 784-8192-8192-10 FP32 DDP (SGD momentum 0.9, per-rank batch 4096)"
METRIC = METRIC_C2
UNIT = "samples/s"


def opt_kwargs(cfg):
    if cfg.optimizer == "adamw":
        return dict(lr=cfg.lr, weight_decay=cfg.weight_decay, betas=cfg.betas, eps=cfg.eps)
    return dict(lr=cfg.lr, momentum=cfg.momentum, dampening=cfg.dampening,
                weight_decay=cfg.weight_decay)


def describe(cfg):
    """'BASELINE configs[i]: MLP ..., optimizer ..., per-rank batch B'."""
    dims = "-".join(str(d) for d in cfg.dims)
    if cfg.optimizer == "adamw":
        opt = f"AdamW lr {cfg.lr:g} wd {cfg.weight_decay:g}"
    else:
        opt = f"SGD momentum {cfg.momentum:g} lr {cfg.lr:g}" if cfg.momentum else f"SGD lr {cfg.lr:g}"
    return f"BASELINE configs[{cfg.name[1:]}]: MLP {dims}, {opt}, per-rank batch {cfg.batch}"


def set_config(name):
    global CFG, METRIC
    CFG = CONFIGS[name]
    METRIC = METRIC_C2 if name == "c2" else (
        f"train samples/s, MLP {'-'.join(str(d) for d in CFG.dims)} FP32 DDP "
        f"({describe(CFG).split(', ', 1)[1]})")


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, limit_s=5.0):
        """Blocks until the first sample has arrived (nvidia-smi takes a
        moment to start, longer with eight processes starting it at once), so
        that a short timed region is still sampled; at most limit_s."""
        t0 = time.perf_counter()
        while self.proc is not None and not self.lines and time.perf_counter() - t0 < limit_s:
            time.sleep(0.01)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _fit(points):
    """Least-squares fixed + per-row cost from (rows, seconds) points."""
    xs = np.array([r for r, _ in points], np.float64)
    ys = np.array([t for _, t in points], np.float64)
    if len(set(xs.tolist())) < 2:
        return None
    per_row, fixed = np.polyfit(xs, ys, 1)
    return {"fixed_s": float(fixed), "per_row_ms": float(per_row * 1e3)}


def cpu_gemm_gflops():
    """GFLOP/s of the timing GEMM (packed FMA kernel, one thread) on a slab
    of the configs' widest product: [256, 8192] x [8192, 1024]."""
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    a = rng.random((256, 8192), dtype=np.float32)
    b = rng.random((8192, 1024), dtype=np.float32)
    O.sgemm_packed(a[:64], b[:, :256])          # page in
    t0 = time.perf_counter()
    ok = O.sgemm_packed(a, b) is not None
    dt = time.perf_counter() - t0
    return 2.0 * 256 * 8192 * 1024 / dt / 1e9 if ok else None


def cpu_step_times(batches):
    """The reference's CPU path (oracle/, restating orca-backend-cpu + the
    Python frontend) timed one step per entry of `batches` (rows per step) on
    the configuration's model: element-wise loops on all host threads (the
    reference's rayon maps), the GEMM single-threaded on the packed FMA
    kernel that stands in for the reference's matrixmultiply (the oracle's
    parity GEMM is a plain loop ~4x slower; it is not what the reference
    runs).  The first step (velocity allocation) is run untimed."""
    from oracle import oracle as O
    O.set_threads(0)
    O.set_gemm_threads(1)
    O.set_gemm_order(4)
    dims = CFG.dims
    kw = opt_kwargs(CFG)
    kw.pop("betas", None), kw.pop("eps", None)
    tr = O.OracleTrainer(dims, init_params(dims, 1), optimizer=CFG.optimizer, **kw)
    xs = {}
    for b in sorted(set(batches)):
        x, t, _ = make_batch(dims, b, 0, CFG.inputs)
        xs[b] = (x, t)
    tr.step(*xs[min(xs)])
    out = []
    for b in batches:
        t0 = time.perf_counter()
        tr.step(*xs[b])
        out.append((b, time.perf_counter() - t0))
    O.set_gemm_order(0)
    return out, O.threads()


def sample_rows():
    """Rows of the CPU samples: 512 and 128, or the configuration's batch and
    a quarter of it when that is smaller."""
    big = min(512, CFG.batch)
    return big, max(1, big // 4)


def cpu_baseline_from(points, cores, label):
    """cpu_baseline object: the measured rate of the largest sample, and the
    fixed + per-row fit of all samples extrapolated to the configuration's
    per-rank batch (the fixed part -- transposes, optimizer passes over every
    parameter -- is paid once per step, so small samples understate the
    reference's rate at the full batch)."""
    fit = _fit(points)
    big = max(r for r, _ in points)
    tb = [t for r, t in points if r == big]
    measured = big / statistics.median(tb)
    full = None
    if fit and fit["per_row_ms"] > 0:
        full = CFG.batch / (max(fit["fixed_s"], 0.0) + CFG.batch * fit["per_row_ms"] / 1e3)
    gf = cpu_gemm_gflops()
    return {"value": full if full else measured, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{label}; value = fixed + per-row fit of the timed steps extrapolated to "
                      f"the {CFG.batch}-row batch (measured {measured:.2f} samples/s at {big} rows)",
            "measured_value": measured, "measured_rows": big,
            "fit": fit, "points": [[r, round(t, 4)] for r, t in points],
            "gemm_gflops": gf,
            "gemm": "packed 8x8 FMA micro-kernel, KC 256 / MC 64 / NC 1024, one thread "
                    "(matrixmultiply 0.3's design, default features)"}


def socket_ddp_baseline(world=2, sample=1 << 20):
    """The reference's socket gradient exchange (oracle/socket_ddp.py restates
    python/orca/distributed.py:65-256: a star through rank 0, Python lists
    averaged in doubles) timed on this host: `world` local processes exchange
    one `sample`-float gradient; the per-step figure scales that to the
    configuration's parameter count (the exchange is linear in the element
    count: byte streams and per-element Python loops)."""
    from oracle import socket_ddp as S
    dt, _, _ = S.run(world, [sample])
    return {"world": world, "sample_floats": sample, "sample_s": dt,
            "per_step_s": dt * CFG.n_params / sample, "kind": "port",
            "sample": f"{world} processes on 127.0.0.1 exchanging one {sample}-float gradient; "
                      f"per step = x {CFG.n_params} / {sample} parameters"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    """The reference arm: the reference's CPU path on the host cores (the
    Rust reference cannot be built here, so its restatement in oracle/ runs),
    rank 0 only.  Warm-up steps run on 128-row samples and timed steps on
    512-row samples (both timed one by one for the fit); `value` is the fit
    extrapolated to the configuration's batch.  At N > 1 every step of the
    reference's DDP job also exchanges every gradient through its socket
    star (timed at world N on this host and added per step)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    big, small = sample_rows()
    pts, cores = cpu_step_times([small] * max(2, args.warmup) + [big] * max(1, args.steps))
    res = cpu_baseline_from(pts, cores, f"{max(1, args.steps)} step(s) at {big} rows and "
                                        f"{max(2, args.warmup)} at {small} rows of the "
                                        f"{'-'.join(str(d) for d in CFG.dims)} {CFG.optimizer} "
                                        f"step: GEMM one thread, element-wise loops on {cores} "
                                        "threads")
    step_s = CFG.batch / res["value"]
    ddp = socket_ddp_baseline(world=args.gpus) if args.gpus > 1 else None
    if ddp:
        step_s += ddp["per_step_s"]
    value = args.gpus * CFG.batch / step_s
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * step_s, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": describe(CFG) + "; CPU; per-rank step time = fixed + per-row "
                                                   f"fit of timed {small}- and {big}-row steps at the "
                                                   f"{CFG.batch}-row batch"
                                                   + (f", plus the socket exchange at world "
                                                      f"{args.gpus}" if ddp else ""),
                       "global_batch": args.gpus * CFG.batch, "per_rank_batch": CFG.batch,
                       "timed_rows_per_step": big,
                       "parallelism": "single process (rank 0)" if args.gpus == 1 else
                       f"rank 0 computes; {args.gpus} ranks assumed, each with the host to itself"},
            "cpu_baseline": dict(res, value=value, socket_ddp=ddp),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)
    return 0


def ddp_parity_check(be, world, rank, dist, local):
    """Data-parallel parity before the timed run (outside it): a reduced
    model (784-1024-1024-10, 512 rows per rank, SGD momentum 0.9, lr 0.01)
    on the tensor-core path through the same trainer and NCCL communicator
    as the timed run, against the oracle's restatement of the reference's
    DDP step (python/orca/distributed.py:238-256: f64 sum over ranks, x 1/W,
    rounded to f32) computed on rank 0 for every rank's batch.
    Step 1 from identical weights: every averaged gradient within 1e-5
    (relative norm) of the oracle's; steps 2-3 run free: per-rank losses
    within 1e-4, parameters within 1e-3 (a ReLU mask flip moves them ~3e-4),
    and every rank's parameters bit-identical."""
    import hashlib
    import torch
    from orcaml_b200.distributed import NcclCommunicator, nccl_unique_id
    from orcaml_b200.mlp import MlpTrainer
    dims, B, steps = [784, 1024, 1024, 10], 512, 3
    kw = dict(lr=0.01, momentum=0.9)
    t0 = time.perf_counter()
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = NcclCommunicator(be, rank, world, obj[0], timeout=120.0)
    tr = MlpTrainer(be, dims, B, optimizer="sgd", gemm_path="tc", **kw)
    tr.set_parameters(init_params(dims, 1))
    tr.attach_comm(comm, bucket_bytes=64 << 20)
    x, t, _ = make_batch(dims, B, rank)
    losses, grads0 = [], None
    for k in range(steps):
        losses.append(tr.step(x, t))
        if k == 0 and rank == 0:
            grads0 = tr.get_grads()
    params = tr.get_parameters()
    digest = hashlib.sha256(b"".join(p.tobytes() for p in params)).hexdigest()
    tr.attach_comm(None)
    comm.close()
    tr.close()
    gathered = [None] * world
    dist.all_gather_object(gathered, (losses, digest))
    out = None
    if rank == 0:
        from oracle import oracle as O
        O.set_threads(0)
        O.set_gemm_threads(0)
        ref = O.OracleTrainer(dims, init_params(dims, 1), optimizer="sgd", **kw)
        batches = [make_batch(dims, B, r) for r in range(world)]
        per = [O.mlp_forward_backward(dims, ref.params, bx, bt) for bx, bt, _ in batches]
        avg = [O.ddp_average([p[1][i] for p in per]) for i in range(len(ref.params))]
        g_err = max(float(np.linalg.norm(g.astype(np.float64) - r) /
                          max(np.linalg.norm(r.astype(np.float64)), 1e-30))
                    for g, r in zip(grads0, avg))
        ref_losses = [[p[0] for p in per]]
        ref.apply(avg)
        for _ in range(steps - 1):
            ref_losses.append(ref.step_ddp([b[0] for b in batches], [b[1] for b in batches]))
        l_err = max(abs(gathered[r][0][k] - ref_losses[k][r]) / abs(ref_losses[k][r])
                    for r in range(world) for k in range(steps))
        p_err = max(float(np.linalg.norm(p.astype(np.float64) - q) /
                          max(np.linalg.norm(q.astype(np.float64)), 1e-30))
                    for p, q in zip(params, ref.params))
        O.set_gemm_threads(1)
        same = len({g[1] for g in gathered}) == 1
        out = {"world": world, "model": "784-1024-1024-10, 512 rows per rank, SGD momentum 0.9, "
                                        "3 steps, tensor-core path",
               "grad_max_rel_err": g_err, "loss_max_rel_err": l_err,
               "param_max_rel_err": p_err, "ranks_identical": same,
               "ok": bool(same and g_err <= 1e-5 and l_err <= 1e-4 and p_err <= 1e-3),
               "seconds": time.perf_counter() - t0}
    torch.cuda.synchronize(local)
    dist.barrier(device_ids=[local])
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from orcaml_b200.backend import CudaBackend
    from orcaml_b200.distributed import NcclCommunicator, nccl_unique_id
    from orcaml_b200.mlp import MlpTrainer

    be = CudaBackend(local)
    parity = None
    if world > 1 and not args.no_parity:
        parity = ddp_parity_check(be, world, rank, dist, local)
    B = CFG.batch
    tr = MlpTrainer(be, CFG.dims, B, optimizer=CFG.optimizer, **opt_kwargs(CFG))
    tr.set_parameters(init_params(CFG.dims, 1))
    comm = None
    if world > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = NcclCommunicator(be, rank, world, obj[0], timeout=120.0)
        tr.attach_comm(comm, bucket_bytes=args.bucket_mb << 20)

    x, t, _ = make_batch(CFG.dims, B, rank, CFG.inputs)
    xs = be.from_f32_slice(list(x.shape), x)
    ts = be.from_f32_slice(list(t.shape), t)
    loss_s = be.zeros([1])
    stream = torch.cuda.ExternalStream(be.stream_handle(), device=torch.device("cuda", local))

    def barrier():
        be.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(local)

    def max_over_ranks(v):
        if world == 1:
            return v
        tt = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    # ---- device-resident step (value) ----
    use_graph = args.graph and world == 1 and CFG.optimizer == "sgd"
    if use_graph:
        tr.graph_capture(xs.device_ptr, ts.device_ptr, loss_s.device_ptr)

    def device_step():
        if use_graph:
            tr.graph_step()
        else:
            tr.step_device(xs.device_ptr, ts.device_ptr, loss_s.device_ptr)

    clocks = ClockSampler(local).__enter__()   # sampling from warm-up on
    clocks.wait_first()
    for _ in range(args.warmup):
        device_step()
    barrier()
    launches0 = be.launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    clocks.lines.clear()                       # keep only samples of the timed region
    barrier()
    ev0.record(stream)
    for _ in range(args.steps):
        device_step()
    ev1.record(stream)
    barrier()
    clocks.__exit__(None, None, None)
    launches = be.launch_count() - launches0
    # The per-kernel breakdown (and the roofline's GEMM time) comes from
    # separate profiled steps after the timed ones, so the profiler's events
    # stay out of `value`.
    if use_graph:
        tr.graph_release()
    prof_steps = max(3, min(args.steps, 10))
    tr.profile_begin()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(prof_steps):
        tr.step_device(xs.device_ptr, ts.device_ptr, loss_s.device_ptr)
    p1.record(stream)
    sites = tr.profile_end()
    barrier()
    prof_ms_step = p0.elapsed_time(p1) / prof_steps
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_step = ms / args.steps
    value = world * B * args.steps / (ms / 1000.0)
    loss_val = float(be.to_f32_vec(loss_s)[0])

    # ---- end to end through the host API: page-locked inputs, H2D + D2H inside ----
    # "staged" (default): the input pipeline -- batch k+1 is copied on the
    # step runner's copy stream while step k computes (two page-locked
    # buffers, two device slots); "step": orca_mlp_step copies, then computes.
    # Either way every step copies its inputs and reads its loss back.
    from orcaml_b200.dataloader import pinned_empty
    bufs = []
    for _ in range(2):
        xp, tp = pinned_empty(x.shape), pinned_empty(t.shape)
        xp[:], tp[:] = x, t
        bufs.append((xp, tp))
    host_loss = ctypes.c_float()

    def e2e_steps(n):
        if args.e2e == "step":
            for _ in range(n):
                tr.step_host_ptr(bufs[0][0].ctypes.data, bufs[0][1].ctypes.data, host_loss)
            return
        tr.stage_batch(0, *bufs[0])
        for k in range(n):
            if k + 1 < n:
                tr.stage_batch((k + 1) % 2, *bufs[(k + 1) % 2])
            tr.step_staged(k % 2)                  # reads the loss back
    e2e_steps(max(1, args.warmup // 2))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * B * args.steps / (e2e_ms / 1000.0)

    # ---- roofline of the dominant kernel: the tcgen05 GEMM ----
    peaks, peak_src = load_peaks()
    tf32_peak = peaks["bf16_tflops"] / 2.0 / 3.0    # FP32-equivalent rate of 3xTF32
    tc_sites = [s for s in sites if s["gemm_path"] == 2]
    tc_ms = sum(s["ms"] for s in tc_sites)
    tc_flops = sum(s["flops"] * s["launches"] for s in tc_sites)
    tc_launches = sum(s["launches"] for s in tc_sites)
    # DRAM read + write of one tcgen05 GEMM launch, from an ncu --set full
    # capture of the configs[2] forward product of the 8192x8192 layer
    # (M=4096, N=8192, K=8192, with the classifier dot; the kDot launch of
    # `python bench.py --steps 3 --warmup 3 --no-cpu`): 2.903 GB read +
    # 0.265 GB written; its algorithmic operand + output bytes are 1.09 GB.
    # Other configs: not captured.
    traffic = {"bytes_per_launch": 3.168e9, "launch": "configs[2] forward 4096x8192x8192 (+dot)",
               "algorithmic_bytes": 1.087e9} if CFG.name == "c2" else None
    achieved = tc_flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else 0.0
    step_flops = CFG.flops_per_sample() * B
    breakdown = {s["name"]: round(s["ms"] / max(1, s["launches"]), 4) for s in sites}

    result = None
    if rank == 0:
        # configs[4]'s CPU step (1.4 B parameters, single-threaded GEMM) would
        # take hours even at 128 rows: not timed.
        cpu = None
        if world == 1 and not args.no_cpu and CFG.name != "c4":
            big, small = sample_rows()
            pts, cores = cpu_step_times([small, big])
            cpu = cpu_baseline_from(pts, cores, f"one step at {small} rows and one at {big} rows of the "
                                    f"{'-'.join(str(d) for d in CFG.dims)} {CFG.optimizer} step: "
                                    f"GEMM one thread, element-wise loops on {cores} threads")
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": f"synthetic ({'uniform [0,1)' if CFG.inputs == 'uniform' else 'N(0,1)'} "
                    "inputs seed=rank, uniform labels, Kaiming-uniform weights seed 1)",
            "config": {"workload": describe(CFG) + (" (device step as a CUDA graph)"
                                                     if use_graph else ""),
                       "global_batch": world * B, "per_rank_batch": B,
                       "parallelism": f"dp{world}",
                       "l2": "working set > L2 (no flush needed)" if CFG.n_params * 16 > 126e6
                       else "working set fits in the 126 MB L2 and is not flushed between steps "
                            "(a reference measurement, not the configs[2] line)",
                       "bucket_mb": args.bucket_mb if world > 1 else None},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": int(x.nbytes + t.nbytes), "d2h_bytes_per_step": 4,
                    "ms_per_step": e2e_ms / args.steps,
                    "pipeline": "copy of batch k+1 overlapped with step k (orca_mlp_stage_batch)"
                    if args.e2e == "staged" else "copy then step (orca_mlp_step)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf32_peak,
                         "unit": "TFLOP/s", "frac": achieved / tf32_peak if tf32_peak else None,
                         "traffic": traffic["bytes_per_launch"] if traffic else None,
                         "traffic_detail": traffic,
                         "kernel": "tc_gemm_kernel (3xTF32 tcgen05, all GEMM launches of the step)",
                         "peak_note": f"{peak_src} bf16 dense {peaks['bf16_tflops']} TFLOP/s / 2 "
                                      "(tf32 rate) / 3 (products per FP32 product)",
                         "launches_per_step": tc_launches / prof_steps,
                         "timing": f"CUDA events around each GEMM launch in {prof_steps} profiled "
                                   "steps run after the timed ones"},
            "step_tflops": step_flops / (ms_step / 1e3) / 1e12,
            "gpu_launches": int(launches),
            "exchange": tr.exchange_kind() if comm is not None else None,
            "loss": loss_val,
            "breakdown_ms": breakdown,
            "breakdown_note": f"per launch, from {prof_steps} profiled steps after the timed ones",
            "profiled_ms_per_step": prof_ms_step,
            "breakdown_sum_ms": sum(s["ms"] for s in sites
                                    if not s["name"].startswith("allreduce")) / prof_steps,
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            result["cpu_baseline"] = dict(cpu, socket_ddp=socket_ddp_baseline())
        if parity is not None:
            result["ddp_parity"] = parity
        print(json.dumps(result), flush=True)
    if comm is not None:
        tr.attach_comm(None)
        comm.close()
    tr.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--bucket-mb", type=int, default=64)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the data-parallel parity pre-check (N > 1)")
    ap.add_argument("--e2e", default="staged", choices=["staged", "step"],
                    help="end-to-end leg: copies overlapped with the previous step, or not")
    ap.add_argument("--graph", action="store_true",
                    help="time the device-resident step as a captured CUDA graph (SGD, N=1)")
    ap.add_argument("--config", default="c2", choices=["c2", "c0", "c1", "c4"],
                    help="BASELINE config (default configs[2], the metric's)")
    args = ap.parse_args()
    set_config(args.config)
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
