"""Data-parallel training on 2 GPUs (one process per GPU, NCCL) vs the oracle.

The oracle restates the reference's DDP step (python/orca/distributed.py:
222-256): each rank's gradients, averaged in f64, then the optimizer.  Each
GPU rank trains on its own seeded batch (seed = rank) with identical initial
weights; after the all-reduce every replica must hold the same parameters
(bit-identical across ranks), and losses/parameters must match the oracle
within 1e-4 relative.  Skipped when fewer than 2 GPUs are visible.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import json, sys
import numpy as np
sys.path.insert(0, REPO)
from orcaml_b200.backend import CudaBackend
from orcaml_b200.mlp import MlpTrainer
from orcaml_b200.distributed import DistributedDataParallel
from orcaml_b200.synthetic import init_params, make_batch
rank, world, port, dims, batch, steps, opt, path = int(sys.argv[1]), int(sys.argv[2]), \
    int(sys.argv[3]), json.loads(sys.argv[4]), int(sys.argv[5]), int(sys.argv[6]), sys.argv[7], \
    sys.argv[8]
be = CudaBackend(rank)
kw = dict(lr=1e-3, weight_decay=0.01) if opt == "adamw" else dict(lr=0.01, momentum=0.9)
tr = MlpTrainer(be, dims, batch, optimizer=opt, gemm_path=path, **kw)
tr.set_parameters(init_params(dims, 1))
ddp = DistributedDataParallel(tr, rank=rank, world_size=world, master_addr=f"127.0.0.1:{port}",
                              timeout=60.0, bucket_bytes=1 << 20)
x, t, _ = make_batch(dims, batch, rank)
losses = [ddp.step(x, t) for _ in range(steps)]
params = tr.get_parameters()
np.savez(OUT + f"/rank{rank}.npz", *params)
json.dump(losses, open(OUT + f"/rank{rank}.json", "w"))
ddp.close()
'''


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("xchg", ["nccl", "peer"])
@pytest.mark.parametrize("opt,dims,batch,path", [("adamw", [784, 256, 256, 10], 64, "auto"),
                                                 ("sgd", [784, 1024, 1024, 10], 512, "tc")])
def test_ddp_two_gpus_matches_oracle(tmp_path, opt, dims, batch, path, xchg):
    """Both exchanges (NCCL all-reduce; the peer-memory kernel).  The "tc"
    case runs the hidden layers on the tensor cores, so with NCCL the dX GEMM
    after each gradient all-reduce is split into two launches (the first on
    fewer CTAs, leaving SMs to the collective)."""
    from oracle import oracle as O
    from orcaml_b200.synthetic import init_params, make_batch
    steps, world, port = 10, 2, 29411 + batch + (0 if xchg == "nccl" else 3)
    code = f"REPO = {REPO!r}\nOUT = {str(tmp_path)!r}\n" + WORKER
    env = dict(os.environ, ORCA_COMM_SMS="16", ORCA_XCHG=xchg)   # exercise the split dX GEMM
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r), str(world), str(port),
                               json.dumps(dims), str(batch), str(steps), opt, path], env=env)
             for r in range(world)]
    try:
        for p in procs:
            assert p.wait(timeout=600) == 0
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait(timeout=60)
    kw = dict(lr=1e-3, weight_decay=0.01) if opt == "adamw" else dict(lr=0.01, momentum=0.9)
    ref = O.OracleTrainer(dims, init_params(dims, 1), optimizer=opt, **kw)
    batches = [make_batch(dims, batch, r) for r in range(world)]
    ref_losses = [ref.step_ddp([b[0] for b in batches], [b[1] for b in batches])
                  for _ in range(steps)]
    finals = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for r in range(world):
        losses = json.load(open(tmp_path / f"rank{r}.json"))
        for s in range(steps):
            assert abs(losses[s] - ref_losses[s][r]) <= 1e-4 * abs(ref_losses[s][r]), (r, s)
    for i, q in enumerate(ref.params):
        p0, p1 = finals[0][f"arr_{i}"], finals[1][f"arr_{i}"]
        assert np.array_equal(p0, p1)          # replicas stay identical
        err = float(np.linalg.norm(p0 - q) / np.linalg.norm(q))
        assert err <= 1e-4, (i, err)


LEAVER = r'''
import json, os, sys, time
sys.path.insert(0, REPO)
from orcaml_b200.backend import CudaBackend
from orcaml_b200.mlp import MlpTrainer
from orcaml_b200.distributed import DistributedDataParallel
from orcaml_b200.synthetic import init_params, make_batch
rank, port, mode = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
dims, B = [784, 256, 256, 10], 64

def wait_for(name, limit=120.0):
    t0 = time.monotonic()
    while not os.path.exists(os.path.join(OUT, name)):
        if time.monotonic() - t0 > limit:
            sys.exit(3)
        time.sleep(0.05)

be = CudaBackend(rank)
tr = MlpTrainer(be, dims, B, optimizer="sgd", lr=0.01, momentum=0.9)
tr.set_parameters(init_params(dims, 1))
ddp = DistributedDataParallel(tr, rank=rank, world_size=2, master_addr=f"127.0.0.1:{port}",
                              timeout=TIMEOUT)
x, t, _ = make_batch(dims, B, rank)
ddp.step(x, t)                                   # both ranks complete step 1
if rank == 1:
    if mode == "exit":
        os._exit(0)                              # leaves between steps, nothing in flight
    wait_for("rank0.done")                       # alive but never joins step 2
    ddp.comm.abort()
    sys.exit(0)
if mode == "exit":
    wait_for("rank1.exited")
t0 = time.monotonic()
try:
    ddp.step(x, t)
    res = {"raised": None}
except RuntimeError as e:
    res = {"raised": str(e)}
res["elapsed"] = time.monotonic() - t0
json.dump(res, open(os.path.join(OUT, "rank0.json"), "w"))
open(os.path.join(OUT, "rank0.done"), "w").close()
ddp.close()
tr.close()
be.close()
'''


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("xchg", ["nccl", "peer"])
@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_ddp_peer_loss_raises_instead_of_hanging(tmp_path, mode, xchg):
    """A peer that exits between steps is seen on the rendezvous sockets before
    the next step launches anything ("exit"); a peer that stays but never joins
    the next step makes the all-reduce miss the 10 s deadline, the
    communicator is aborted ("stall"); with the peer exchange the survivor's
    kernel gives up its bounded wait for the peer's ready flag.  Either way the surviving rank gets
    RuntimeError, well before any outer bound, and exits cleanly.  NVLS is off
    (NCCL_NVLS_ENABLE=0) so no rank's memory is bound to a multicast object."""
    port = 29611 + (0 if mode == "exit" else 7) + (0 if xchg == "nccl" else 20)
    code = f"REPO = {REPO!r}\nOUT = {str(tmp_path)!r}\nTIMEOUT = 10.0\n" + LEAVER
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", ORCA_XCHG=xchg)
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r), str(port), mode], env=env)
             for r in range(2)]
    try:
        if mode == "exit":
            assert procs[1].wait(timeout=120) == 0
            (tmp_path / "rank1.exited").touch()
        assert procs[0].wait(timeout=120) == 0
        assert procs[1].wait(timeout=120) == 0
    finally:
        for p in procs:          # never leave a rank behind holding a GPU
            if p.poll() is None:
                p.kill()
                p.wait(timeout=60)
    res = json.load(open(tmp_path / "rank0.json"))
    assert res["raised"] is not None
    if mode == "exit":
        assert "closed its connection" in res["raised"] and res["elapsed"] < 5.0
    else:
        assert "stopped responding" in res["raised"] and 9.0 <= res["elapsed"] < 60.0


EXACT = r"""
import json, sys
import numpy as np
sys.path.insert(0, REPO)
from orcaml_b200.backend import CudaBackend
from orcaml_b200.mlp import MlpTrainer
from orcaml_b200.distributed import DistributedDataParallel
from orcaml_b200.synthetic import init_params, make_batch
rank, world, port, xchg = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
dims, B = [784, 1024, 1024, 10], 512
be = CudaBackend(rank)
x, t, _ = make_batch(dims, B, rank)
solo = MlpTrainer(be, dims, B, optimizer="sgd", lr=0.0, gemm_path="tc")
solo.set_parameters(init_params(dims, 1))
solo.step(x, t)
np.savez(OUT + f"/local{rank}.npz", *solo.get_grads())
solo.close()
tr = MlpTrainer(be, dims, B, optimizer="sgd", lr=0.0, gemm_path="tc")
tr.set_exchange(xchg)
tr.set_parameters(init_params(dims, 1))
ddp = DistributedDataParallel(tr, rank=rank, world_size=world, master_addr=f"127.0.0.1:{port}",
                              timeout=60.0)
for _ in range(3):                    # lr 0: the same gradients every step
    ddp.step(x, t)
kind = tr.exchange_kind()
np.savez(OUT + f"/avg{rank}.npz", *tr.get_grads())
json.dump(kind, open(OUT + f"/kind{rank}.json", "w"))
ddp.close()
"""


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("xchg", ["nccl", "peer"])
def test_exchange_is_the_reference_average_bit_for_bit(tmp_path, xchg):
    """Each rank's averaged gradients equal, bit for bit, the reference's
    average (python/orca/distributed.py:238-256: float64 sum in rank order,
    x 1/world, rounded to float32; oracle.ddp_average) of the ranks' own local
    gradients (computed by a trainer without a communicator: the kernels are
    deterministic, so they are the gradients the exchange received), on three
    consecutive steps (the peer exchange's sequence numbers advance)."""
    from oracle import oracle as O
    world, port = 2, 29711 + (0 if xchg == "nccl" else 5)
    code = f"REPO = {REPO!r}\nOUT = {str(tmp_path)!r}\n" + EXACT
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r), str(world), str(port), xchg],
                              env=env) for r in range(world)]
    try:
        for p in procs:
            assert p.wait(timeout=600) == 0
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait(timeout=60)
    local = [np.load(tmp_path / f"local{r}.npz") for r in range(world)]
    avg = [np.load(tmp_path / f"avg{r}.npz") for r in range(world)]
    for r in range(world):
        assert json.load(open(tmp_path / f"kind{r}.json")) == xchg
    for i in range(len(local[0].files)):
        ref = O.ddp_average([local[r][f"arr_{i}"] for r in range(world)])
        for r in range(world):
            assert np.array_equal(avg[r][f"arr_{i}"], ref), (i, r)
