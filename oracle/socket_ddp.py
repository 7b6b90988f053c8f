"""The reference's socket gradient exchange, restated for timing on the host.

TEST / BASELINE INFRASTRUCTURE ONLY: bench.py's CPU-baseline leg runs it to
time the reference's data-parallel exchange on the machine's own cores, and
tests/ check its arithmetic against oracle.ddp_average.  The product package
never imports it.

What it restates (python/orca/distributed.py):
  * rendezvous (:160-212): rank 0 listens, accepts world-1 connections with
    TCP_NODELAY; the other ranks retry connect until a deadline;
  * framing (:65-117): an 8-byte big-endian element count ("!Q"), then the
    values as big-endian float32 ("!{n}f"), a length mismatch is an error;
  * all_reduce_gradients (:222-256), per parameter: the gradient becomes a
    Python list (`to_list`); rank 0 adds every peer's list element by element
    into Python floats (f64), multiplies each sum by 1/world_size (f64) and
    sends the result back, which the "!f" packing rounds to float32; every
    rank then builds its tensor from that list (`from_list`, float32).
The exchange runs through rank 0 (a star): rank 0 receives and sends
(world-1) x the gradient bytes, and the per-element work is Python loops.
"""
from __future__ import annotations

import multiprocessing as mp
import socket
import struct
import time
from typing import List, Sequence

import numpy as np

COUNT_FORMAT = "!Q"
COUNT_BYTES = struct.calcsize(COUNT_FORMAT)


def _recv_exact(conn: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = conn.recv(n - len(buf))
        if not chunk:
            raise RuntimeError(f"peer closed after {len(buf)} of {n} bytes")
        buf.extend(chunk)
    return bytes(buf)


def _send_values(conn: socket.socket, values: List[float]) -> None:
    conn.sendall(struct.pack(COUNT_FORMAT, len(values)))
    if values:
        conn.sendall(struct.pack(f"!{len(values)}f", *values))


def _recv_values(conn: socket.socket, expected: int) -> List[float]:
    (n,) = struct.unpack(COUNT_FORMAT, _recv_exact(conn, COUNT_BYTES))
    if n != expected:
        raise RuntimeError(f"gradient size mismatch: expected {expected}, got {n}")
    if n == 0:
        return []
    return list(struct.unpack(f"!{n}f", _recv_exact(conn, 4 * n)))


def exchange(rank: int, world: int, conns: Sequence[socket.socket],
             grads: Sequence[np.ndarray]) -> List[np.ndarray]:
    """One all_reduce_gradients call over established connections (rank 0:
    one connection per peer; others: the connection to rank 0)."""
    inv = 1.0 / world
    out = []
    for g in grads:
        data = np.asarray(g, np.float32).reshape(-1).tolist()      # grad.to_list()
        n = len(data)
        if rank == 0:
            total = list(data)
            for conn in conns:
                for i, v in enumerate(_recv_values(conn, n)):
                    total[i] += v
            avg = [v * inv for v in total]
            for conn in conns:
                _send_values(conn, avg)
        else:
            _send_values(conns[0], data)
            avg = _recv_values(conns[0], n)
        out.append(np.asarray(avg, np.float64).astype(np.float32).reshape(np.shape(g)))
    return out


def connect(rank: int, world: int, port: int, timeout: float = 30.0) -> List[socket.socket]:
    if rank == 0:
        conns = []
        with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as srv:
            srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            srv.settimeout(timeout)
            srv.bind(("127.0.0.1", port))
            srv.listen(world - 1)
            for _ in range(1, world):
                c, _ = srv.accept()
                c.settimeout(timeout)
                c.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
                conns.append(c)
        return conns
    deadline = time.monotonic() + timeout
    while True:
        c = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        c.settimeout(min(1.0, timeout))
        c.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        try:
            c.connect(("127.0.0.1", port))
            c.settimeout(timeout)
            return [c]
        except OSError:
            c.close()
            if time.monotonic() > deadline:
                raise
            time.sleep(0.05)


def _peer(rank, world, port, sizes, seed, q):
    try:
        conns = connect(rank, world, port)
        rng = np.random.default_rng(seed + rank)
        grads = [rng.standard_normal(n).astype(np.float32) for n in sizes]
        out = exchange(rank, world, conns, grads)
        q.put((rank, [o.tobytes() for o in out]))
        for c in conns:
            c.close()
    except BaseException as exc:  # reported to the parent
        q.put((rank, repr(exc)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run(world: int, sizes: Sequence[int], seed: int = 0, timeout: float = 120.0):
    """Rank 0 in this process, ranks 1.. as spawned processes on 127.0.0.1.
    Returns (seconds rank 0 spent in the exchange, rank 0's averaged
    gradients, every rank's inputs)."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    q = ctx.Queue()
    procs = [ctx.Process(target=_peer, args=(r, world, port, list(sizes), seed, q), daemon=True)
             for r in range(1, world)]
    for p in procs:
        p.start()
    try:
        conns = connect(0, world, port, timeout)
        rng = np.random.default_rng(seed)
        grads = [rng.standard_normal(n).astype(np.float32) for n in sizes]
        t0 = time.perf_counter()
        out = exchange(0, world, conns, grads)
        dt = time.perf_counter() - t0
        for c in conns:
            c.close()
        for _ in procs:
            rank, res = q.get(timeout=timeout)
            if isinstance(res, str):
                raise RuntimeError(f"rank {rank}: {res}")
    finally:
        for p in procs:
            p.join(timeout=10.0)
            if p.is_alive():
                p.kill()
    inputs = []
    for r in range(world):
        rng = np.random.default_rng(seed + r)
        inputs.append([rng.standard_normal(n).astype(np.float32) for n in sizes])
    return dt, out, inputs
