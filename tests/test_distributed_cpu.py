"""Host side of the data-parallel path, on CPU with 2 processes (no GPU).

* the NCCL-id rendezvous keeps the reference's TCP topology and failure
  behaviour (python/orca/distributed.py:161-210): rank 0 listens, workers
  retry until a deadline, everyone gets rank 0's 128-byte id;
* argument validation raises the reference's TypeError/ValueError
  (distributed.py:19-62, python/tests/test_phase8.py:60-106);
* a rank that never joins makes the others fail with RuntimeError after the
  timeout instead of hanging; a rank that leaves after joining is seen on
  the kept rendezvous sockets before the next step;
* the bench's plumbing over torch.distributed `gloo`, world 2: the id
  broadcast and the max-over-ranks timing reduction.
"""
import multiprocessing as mp
import os
import socket

import pytest

from orcaml_b200 import distributed as D


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(rank, world, addr, q):
    try:
        got = D.exchange_id(rank, world, addr, 20.0, lambda: bytes(range(128)))
        q.put((rank, got))
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put((rank, repr(e)))


def test_rendezvous_two_ranks_get_rank0_id():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    addr = f"127.0.0.1:{_free_port()}"
    ps = [ctx.Process(target=_exchange, args=(r, 2, addr, q)) for r in (1, 0)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in ps:
        p.join(30)
    assert res[0] == bytes(range(128)) and res[1] == bytes(range(128))


def test_rendezvous_missing_peer_times_out():
    addr = f"127.0.0.1:{_free_port()}"
    with pytest.raises(RuntimeError):
        D.exchange_id(1, 2, addr, 1.0, lambda: bytes(128))   # nobody listens
    with pytest.raises(RuntimeError):
        D.exchange_id(0, 2, addr, 1.0, lambda: bytes(128))   # nobody connects


def _leaver(addr, q):
    payload, links = D.rendezvous(1, 2, addr, 20.0, lambda: bytes(128))
    links.check()                     # rank 0 still there
    q.put("joined")
    links.close()                     # leave between steps


def test_peer_links_report_a_rank_that_left():
    """The rendezvous sockets stay open as the liveness channel: while the
    worker is there check() passes; after it closes its end (or exits),
    rank 0's next check() raises RuntimeError -- before any collective."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    addr = f"127.0.0.1:{_free_port()}"
    p = ctx.Process(target=_leaver, args=(addr, q))
    p.start()
    payload, links = D.rendezvous(0, 2, addr, 20.0, lambda: bytes(range(128)))
    assert payload == bytes(range(128))
    links.check()
    assert q.get(timeout=60) == "joined"
    p.join(30)
    assert p.exitcode == 0
    with pytest.raises(RuntimeError, match="closed its connection"):
        links.check()
    links.close()


@pytest.mark.parametrize("rank,world,exc", [(True, 2, TypeError), (0, "2", TypeError),
                                            (0, 0, ValueError), (2, 2, ValueError),
                                            (-1, 2, ValueError)])
def test_process_group_validation(rank, world, exc):
    with pytest.raises(exc):
        D._validate_process_group(rank, world)


@pytest.mark.parametrize("addr,exc", [("nohost", ValueError), (":80", ValueError),
                                      ("h:x", ValueError), ("h:0", ValueError),
                                      ("h:70000", ValueError), (5, TypeError)])
def test_master_addr_validation(addr, exc):
    with pytest.raises(exc):
        D._parse_master_addr(addr)


@pytest.mark.parametrize("timeout,exc", [(0, ValueError), (-1.0, ValueError),
                                         (True, TypeError), ("x", TypeError)])
def test_timeout_validation(timeout, exc):
    with pytest.raises(exc):
        D._validate_timeout(timeout)


def _gloo_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    obj = [bytes([7] * 128) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    t = torch.tensor([float(10 + rank)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    q.put((rank, obj[0], float(t.item())))
    dist.destroy_process_group()


def test_bench_plumbing_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (uid, mx)) for r, uid, mx in (q.get(timeout=120) for _ in range(2)))
    for p in ps:
        p.join(60)
    for r in range(2):
        assert res[r][0] == bytes([7] * 128)   # the NCCL id reaches every rank
        assert res[r][1] == 11.0               # max over ranks


def test_allreduce_sweep_needs_two_ranks(capsys, monkeypatch):
    """The sweep module loads without a GPU and declines a single rank."""
    import json as _json
    from orcaml_b200 import allreduce_sweep
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    assert allreduce_sweep.main([]) == 0
    assert "skipped" in _json.loads(capsys.readouterr().out.strip().splitlines()[-1])
