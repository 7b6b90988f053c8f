"""Gradient all-reduce sweep (north-star configs[3]): flat f32 buffers from
1 MB to 1 GB in powers of two, N(0,1) values drawn with seed = rank, averaged
in place across the ranks by the library's communicator (orca_comm_*: one
NCCL all-reduce with ncclAvg per bucket), reporting bus GB/s.

The reference's exchange for the same job is the TCP star of
python/orca/distributed.py:222-256 (every rank ships its gradients to rank 0,
which averages them in Python doubles and sends the mean back); here the
buffers never leave the GPUs.

Run one process per GPU:

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port P -m orcaml_b200.allreduce_sweep

Per size: 3 untimed calls, then `iters` calls timed with CUDA events on the
library's compute stream (each call is ordered after it and the stream waits
for the call to finish), max over ranks.  bus GB/s = 2 (n-1)/n * bytes / time,
the traffic each rank's link carries in a ring or tree all-reduce; it is
compared with the measured one-way peer copy bandwidth of this pool's
NVLink (770 GB/s).  Before timing, the first 4 Mi elements of one freshly
filled buffer are checked against the float64 average of every rank's
values (regenerated locally from the seeds).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

PEER_COPY_GBS = 770.0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-mb", type=int, default=1)
    ap.add_argument("--max-mb", type=int, default=1024)
    ap.add_argument("--bucket-mb", type=int, default=0,
                    help="split each buffer into all-reduce calls of this size (0 = one call)")
    ap.add_argument("--out", default=None, help="also write the JSON line here (rank 0)")
    args = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print(json.dumps({"metric": "allreduce bus GB/s", "skipped": "needs >= 2 ranks"}))
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from orcaml_b200.backend import CudaBackend
    from orcaml_b200.distributed import NcclCommunicator, nccl_unique_id

    be = CudaBackend(local)
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = NcclCommunicator(be, rank, world, obj[0], timeout=120.0)
    stream = torch.cuda.ExternalStream(be.stream_handle(), device=dev)

    max_elems = (args.max_mb << 20) // 4
    buf = torch.empty(max_elems, dtype=torch.float32, device=dev)

    def fill(n):
        g = torch.Generator(device=dev)
        g.manual_seed(rank)
        buf[:n].normal_(generator=g)
        torch.cuda.synchronize(dev)

    def allreduce(n):
        ptr = buf.data_ptr()
        chunk = (args.bucket_mb << 20) // 4 if args.bucket_mb else n
        for off in range(0, n, chunk):
            comm.allreduce_avg(ptr + 4 * off, min(chunk, n - off))

    def barrier():
        be.synchronize()
        dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        tt = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    # ---- correctness: one average of freshly filled buffers vs float64 ----
    n_chk = min(max_elems, 4 << 20)
    fill(n_chk)
    barrier()
    allreduce(n_chk)
    barrier()
    got = buf[:n_chk].double()
    acc = torch.zeros(n_chk, dtype=torch.float64, device=dev)
    mag = torch.zeros(n_chk, dtype=torch.float64, device=dev)
    for r in range(world):
        g = torch.Generator(device=dev)
        g.manual_seed(r)
        v = torch.empty(n_chk, dtype=torch.float32, device=dev).normal_(generator=g).double()
        acc += v
        mag += v.abs()
    ref = acc / world
    err = (got - ref).abs()
    # f32 summation of `world` terms then one scaling: a few ulp of the sum's magnitude.
    bound = (world + 2) * 2.0 ** -24 * mag / world + 1e-30
    check = {"elements": n_chk, "max_abs_err": float(err.max()),
             "max_err_over_bound": float((err / bound).max()),
             "ok": bool((err <= bound).all())}
    check["ok"] = max_over_ranks(0.0 if check["ok"] else 1.0) == 0.0

    # ---- timing ----
    rows = []
    mb = args.min_mb
    fill(max_elems)
    while mb <= args.max_mb:
        n = (mb << 20) // 4
        iters = 20 if mb <= 64 else (10 if mb <= 256 else 5)
        for _ in range(3):
            allreduce(n)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            allreduce(n)
        e1.record(stream)
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / iters
        size = n * 4
        busbw = 2.0 * (world - 1) / world * size / (ms / 1e3) / 1e9
        rows.append({"bytes": size, "ms": round(ms, 5),
                     "algbw_gbs": round(size / (ms / 1e3) / 1e9, 2),
                     "busbw_gbs": round(busbw, 2),
                     "frac_of_peer_copy": round(busbw / PEER_COPY_GBS, 4)})
        mb *= 2

    if rank == 0:
        line = {"metric": "allreduce bus GB/s (ncclAvg, in place, f32)", "n_gpus": world,
                "config": {"workload": "BASELINE configs[3]: flat f32 buffers "
                                       f"{args.min_mb} MB..{args.max_mb} MB, N(0,1) seed=rank",
                           "bucket_mb": args.bucket_mb or None},
                "peak": {"value": PEER_COPY_GBS, "unit": "GB/s",
                         "what": "measured NVLink peer copy per direction on this pool"},
                "check": check, "sizes": rows,
                "busbw_at_max_gbs": rows[-1]["busbw_gbs"] if rows else None}
        s = json.dumps(line)
        print(s, flush=True)
        if args.out:
            with open(args.out, "w") as f:
                f.write(s + "\n")
    barrier()
    comm.close()
    be.close()
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    return 0 if check["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
