"""Generate the golden fixtures in tests/golden/ from the reference's own Python.

Run in the development container, where the reference source tree is mounted:

    python tests/golden/make_golden.py /path/to/reference/python

The reference's Python frontend (python/orca/nn, optim, distributed) is pure
Python over the compiled `orca.orca_python` module, which cannot be built here
(no Rust toolchain).  oracle/orca_shim.py provides that module from the
restated CPU backend + tape autograd, and this script drives the reference's
unchanged Sequential/Linear/ReLU/CrossEntropyLoss/SGD/AdamW/
DistributedDataParallel code on top of it -- the op composition and the
constants therefore come from the reference itself.  Each case is also run
through the fused oracle step (oracle/oracle.py OracleTrainer) and the script
refuses to write a fixture unless both agree bit for bit.

Fixtures hold loss traces as exact float32 bit patterns, SHA-256 digests and
checksums of the final parameters, final argmax predictions, and (for the
small cases) the full final parameters.
"""
from __future__ import annotations

import hashlib
import json
import multiprocessing as mp
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402
from orcaml_b200.synthetic import init_params, make_batch  # noqa: E402

STEPS = 20


def f32_bits(v) -> str:
    return np.float32(v).view(np.uint32).tobytes().hex()


def params_digest(params) -> str:
    h = hashlib.sha256()
    for p in params:
        h.update(np.ascontiguousarray(p, dtype=np.float32).tobytes())
    return h.hexdigest()


def summary(params):
    return {
        "sha256": params_digest(params),
        "sum": [float(np.sum(p, dtype=np.float64)) for p in params],
        "abs_sum": [float(np.sum(np.abs(p), dtype=np.float64)) for p in params],
        "first8": [[float(v) for v in p.reshape(-1)[:8]] for p in params],
    }


def _reference_model(orca, dims, params):
    nn = orca.nn
    layers = []
    for i in range(len(dims) - 1):
        layers.append(nn.Linear(dims[i], dims[i + 1]))
        if i + 2 < len(dims):
            layers.append(nn.ReLU())
    model = nn.Sequential(*layers)
    for p, arr in zip(model.parameters(), params):
        p.update(orca.Tensor.from_list(arr.reshape(-1), shape=list(arr.shape), requires_grad=True))
    return model


def _make_opt(orca, model, case):
    if case["optimizer"] == "sgd":
        return orca.optim.SGD(model.parameters(), lr=case["lr"], momentum=case.get("momentum", 0.0))
    return orca.optim.AdamW(model.parameters(), lr=case["lr"], weight_decay=case["weight_decay"])


def run_reference_single(ref_dir, case):
    from oracle import orca_shim
    orca = orca_shim.install(ref_dir)
    dims = case["dims"]
    params = init_params(dims, 1)
    x, t, _ = make_batch(dims, case["batch"], 0)
    model = _reference_model(orca, dims, params)
    opt = _make_opt(orca, model, case)
    loss_fn = orca.nn.CrossEntropyLoss()
    X = orca.Tensor.from_list(x.reshape(-1), shape=list(x.shape))
    T = orca.Tensor.from_list(t.reshape(-1), shape=list(t.shape))
    losses = []
    for _ in range(STEPS):
        opt.zero_grad()
        pred = model(X)
        loss = loss_fn(pred, T)
        loss.backward()
        opt.step()
        losses.append(np.float32(loss.to_list()[0]))
    final = [np.asarray(p.tensor.to_list(), np.float32).reshape(a.shape)
             for p, a in zip(model.parameters(), params)]
    with orca.no_grad():
        logits = np.asarray(model(X).to_list(), np.float32).reshape(x.shape[0], dims[-1])
    return losses, final, logits


def _ddp_worker(ref_dir, case, rank, world, addr, q):
    sys.path.insert(0, REPO)
    from oracle import orca_shim
    orca = orca_shim.install(ref_dir)
    from orca.distributed import DistributedDataParallel
    dims = case["dims"]
    params = init_params(dims, 1)
    x, t, _ = make_batch(dims, case["batch"], rank)
    model = _reference_model(orca, dims, params)
    ddp = DistributedDataParallel(model, rank=rank, world_size=world, master_addr=addr, timeout=120)
    opt = _make_opt(orca, ddp, case)
    loss_fn = orca.nn.CrossEntropyLoss()
    X = orca.Tensor.from_list(x.reshape(-1), shape=list(x.shape))
    T = orca.Tensor.from_list(t.reshape(-1), shape=list(t.shape))
    losses = []
    try:
        for _ in range(STEPS):
            opt.zero_grad()
            loss = loss_fn(ddp(X), T)
            loss.backward()
            ddp.all_reduce_gradients()
            opt.step()
            losses.append(float(np.float32(loss.to_list()[0])))
        final = [np.asarray(p.tensor.to_list(), np.float32).reshape(a.shape)
                 for p, a in zip(ddp.parameters(), params)]
        q.put((rank, losses, [f.tolist() for f in final]))
    finally:
        ddp.close()


def run_reference_ddp(ref_dir, case, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = case["world"]
    procs = [ctx.Process(target=_ddp_worker, args=(ref_dir, case, r, world, f"127.0.0.1:{port}", q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, losses, final = q.get(timeout=3600)
        res[r] = (losses, [np.asarray(f, np.float32) for f in final])
    for p in procs:
        p.join()
    return res


def run_oracle(case, ranks):
    dims = case["dims"]
    tr = O.OracleTrainer(dims, init_params(dims, 1), optimizer=case["optimizer"], lr=case["lr"],
                         momentum=case.get("momentum", 0.0),
                         weight_decay=case.get("weight_decay", 0.0))
    batches = [make_batch(dims, case["batch"], r) for r in range(ranks)]
    losses = [[] for _ in range(ranks)]
    for _ in range(STEPS):
        if ranks == 1:
            losses[0].append(np.float32(tr.step(batches[0][0], batches[0][1])))
        else:
            for r, l in enumerate(tr.step_ddp([b[0] for b in batches], [b[1] for b in batches])):
                losses[r].append(np.float32(l))
    _, logits = O.mlp_forward(dims, tr.params, batches[0][0], batches[0][1])
    return losses, tr.params, logits


CASES = [
    # BASELINE.json configs[0] exactly: 784-512-512-10, B=128, SGD lr 0.1, 20 steps.
    {"name": "c0", "dims": [784, 512, 512, 10], "batch": 128, "optimizer": "sgd", "lr": 0.1,
     "full_params": False},
    # configs[2]'s optimizer (SGD momentum 0.9, lr 0.01) on a small MLP, full params kept.
    {"name": "sgdm_small", "dims": [24, 20, 12, 10], "batch": 16, "optimizer": "sgd", "lr": 0.01,
     "momentum": 0.9, "full_params": True},
    {"name": "sgd_small", "dims": [32, 16, 16, 10], "batch": 8, "optimizer": "sgd", "lr": 0.1,
     "full_params": True},
    # configs[1]'s recipe (AdamW lr 1e-3 wd 0.01, socket DDP world 2) at reduced width.
    {"name": "adamw_ddp2_small", "dims": [40, 24, 24, 10], "batch": 12, "optimizer": "adamw",
     "lr": 1e-3, "weight_decay": 0.01, "world": 2, "full_params": True},
    {"name": "c1_ddp2_mid", "dims": [784, 256, 256, 10], "batch": 64, "optimizer": "adamw",
     "lr": 1e-3, "weight_decay": 0.01, "world": 2, "full_params": False},
]


def ce_cases(ref_dir):
    """Softmax-CE forward/backward through the reference's CrossEntropyLoss on
    inputs with ties at the row max and a non-one-hot target row."""
    from oracle import orca_shim
    orca = orca_shim.install(ref_dir)
    P = np.array([[1.0, 3.0, 3.0, -2.0],     # tie at the max
                  [0.5, 0.5, 0.5, 0.5],      # all tied
                  [-1e3, 2.0, 7.5, 7.25],
                  [10.0, -10.0, 0.0, 1e-3]], np.float32)
    T = np.array([[0, 1, 0, 0],
                  [0, 0, 0, 1],
                  [0.25, 0.25, 0.5, 0],      # soft target
                  [1, 0, 0, 0]], np.float32)
    p = orca.Tensor.from_list(P.reshape(-1), shape=[4, 4], requires_grad=True)
    t = orca.Tensor.from_list(T.reshape(-1), shape=[4, 4])
    loss = orca.nn.CrossEntropyLoss()(p, t)
    loss.backward()
    dP = np.asarray(p.grad().to_list(), np.float32).reshape(4, 4)
    lo, dPo = O.softmax_ce(P, T)
    assert np.float32(loss.to_list()[0]).tobytes() == np.float32(lo).tobytes(), "CE loss mismatch"
    assert np.array_equal(dP, dPo), (dP, dPo)
    return {"P": P.tolist(), "T": T.tolist(), "loss_bits": f32_bits(loss.to_list()[0]),
            "dP_bits": [f32_bits(v) for v in dP.reshape(-1)]}


def main(ref_dir):
    out = {}
    port = 19931
    for case in CASES:
        world = case.get("world", 1)
        if world == 1:
            ref_losses, ref_final, ref_logits = run_reference_single(ref_dir, case)
            ref_losses = [ref_losses]
        else:
            res = run_reference_ddp(ref_dir, case, port)
            port += 1
            ref_losses = [res[r][0] for r in range(world)]
            ref_final = res[0][1]
            for r in range(1, world):
                assert params_digest(res[r][1]) == params_digest(ref_final), "replicas diverged"
            ref_logits = None
        or_losses, or_final, or_logits = run_oracle(case, world)
        for r in range(world):
            a = [f32_bits(v) for v in ref_losses[r]]
            b = [f32_bits(v) for v in or_losses[r]]
            assert a == b, f"{case['name']}: loss trace differs on rank {r}\n{a}\n{b}"
        assert params_digest(ref_final) == params_digest(or_final), f"{case['name']}: params differ"
        if ref_logits is not None:
            assert np.array_equal(ref_logits, or_logits)
        rec = {k: v for k, v in case.items() if k != "full_params"}
        rec["steps"] = STEPS
        rec["loss_bits"] = [[f32_bits(v) for v in l] for l in ref_losses]
        rec["final"] = summary(ref_final)
        rec["argmax"] = [int(v) for v in np.argmax(or_logits, axis=1)]
        out[case["name"]] = rec
        if case["full_params"]:
            np.savez(os.path.join(HERE, f"{case['name']}_final.npz"),
                     *[np.asarray(p, np.float32) for p in ref_final])
        print(f"{case['name']}: reference == fused oracle, loss {ref_losses[0][0]:.6f} -> "
              f"{ref_losses[0][-1]:.6f}")
    out["ce_ties"] = ce_cases(ref_dir)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference>/python")
    main(sys.argv[1])
