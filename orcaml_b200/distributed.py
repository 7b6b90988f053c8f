"""Data-parallel gradient exchange over NCCL, with the reference's DDP surface.

The reference's `DistributedDataParallel` (python/orca/distributed.py:127-256)
rendezvous over TCP (rank 0 listens on master_addr, workers retry until a
deadline, :161-210) and then ships every gradient through rank 0 as Python
lists.  Here the same rendezvous only ships the 128-byte NCCL unique id; the
gradients never leave the GPUs: each layer's (dW, db) is all-reduced with
fused averaging (ncclAvg) on a side stream as soon as the backward pass has
produced it (orca_mlp_attach_comm).  Argument validation and error behaviour
(TypeError/ValueError for bad arguments, RuntimeError for rendezvous
failures) follow the reference's helpers (:19-62).
"""
from __future__ import annotations

import ctypes
import socket
import time

from . import _lib as L

_DEFAULT_TIMEOUT_SECONDS = 30.0
ID_BYTES = 128


def _validate_timeout(timeout) -> float:
    if isinstance(timeout, bool):
        raise TypeError("timeout must be a positive number")
    try:
        value = float(timeout)
    except (TypeError, ValueError) as exc:
        raise TypeError("timeout must be a positive number") from exc
    if value <= 0.0:
        raise ValueError("timeout must be positive")
    return value


def _validate_process_group(rank, world_size) -> None:
    if isinstance(rank, bool) or not isinstance(rank, int):
        raise TypeError("rank must be an integer")
    if isinstance(world_size, bool) or not isinstance(world_size, int):
        raise TypeError("world_size must be an integer")
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    if rank < 0 or rank >= world_size:
        raise ValueError(f"rank must be in [0, {world_size})")


def _parse_master_addr(master_addr):
    if not isinstance(master_addr, str):
        raise TypeError("master_addr must be a string in 'host:port' format")
    try:
        host, port_text = master_addr.rsplit(":", 1)
    except ValueError as exc:
        raise ValueError("master_addr must use 'host:port' format") from exc
    if not host:
        raise ValueError("master_addr host cannot be empty")
    try:
        port = int(port_text)
    except ValueError as exc:
        raise ValueError("master_addr port must be an integer") from exc
    if port <= 0 or port > 65535:
        raise ValueError("master_addr port must be in the range [1, 65535]")
    return host, port


def _recv_exact(conn: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        try:
            chunk = conn.recv(n - len(buf))
        except socket.timeout as exc:
            raise RuntimeError(f"Timed out while reading {n} bytes from distributed peer") from exc
        except OSError as exc:
            raise RuntimeError("Failed to read from distributed peer") from exc
        if not chunk:
            raise RuntimeError(f"Distributed peer closed connection after {len(buf)} of {n} bytes")
        buf.extend(chunk)
    return bytes(buf)


class PeerLinks:
    """The rendezvous sockets, kept open as a liveness channel.

    Rank 0 holds one connection per worker, each worker one to rank 0 (the
    reference's star, python/orca/distributed.py:161-210).  Nothing is sent on
    them after the rendezvous, so a readable socket means its peer closed it
    or exited: `check()` raises RuntimeError before the next step launches any
    collective that the peer would never join."""

    def __init__(self, rank: int, conns):
        self.rank = rank
        self.conns = list(conns)

    def check(self):
        import select
        if not self.conns:
            return
        readable, _, errored = select.select(self.conns, [], self.conns, 0)
        for conn in set(readable) | set(errored):
            try:
                data = conn.recv(1, socket.MSG_PEEK)
            except OSError:
                data = b""
            if not data:
                raise RuntimeError(f"Rank {self.rank}: distributed peer closed its connection")

    def close(self):
        for conn in self.conns:
            try:
                conn.close()
            except OSError:
                pass
        self.conns = []


def rendezvous(rank: int, world_size: int, master_addr: str, timeout: float, make_id):
    """Rank 0 calls make_id() and sends the bytes to every worker over TCP;
    returns (id bytes, PeerLinks holding the open connections).

    Same topology and failure behaviour as the reference's _connect: rank 0
    binds and accepts world_size-1 peers within `timeout`; workers retry the
    connection until the deadline."""
    host, port = _parse_master_addr(master_addr)
    if world_size == 1:
        return make_id(), PeerLinks(rank, [])
    if rank == 0:
        payload = make_id()
        if len(payload) != ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        peers = []
        try:
            with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as srv:
                srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
                srv.settimeout(timeout)
                srv.bind((host, port))
                srv.listen(world_size - 1)
                for _ in range(1, world_size):
                    conn, _ = srv.accept()
                    conn.settimeout(timeout)
                    peers.append(conn)
                for conn in peers:
                    conn.sendall(payload)
                for conn in peers:       # wait for every worker's acknowledgement
                    if _recv_exact(conn, 1) != b"\x01":
                        raise RuntimeError("bad acknowledgement from distributed peer")
        except (OSError, RuntimeError) as exc:
            PeerLinks(rank, peers).close()
            if isinstance(exc, RuntimeError):
                raise
            raise RuntimeError(f"Rank 0 failed to initialize distributed listener at {master_addr}") from exc
        return payload, PeerLinks(rank, peers)
    deadline = time.monotonic() + timeout
    last = None
    while time.monotonic() < deadline:
        cli = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        cli.settimeout(min(1.0, timeout))
        try:
            cli.connect((host, port))
            cli.settimeout(max(0.001, deadline - time.monotonic()))
            payload = _recv_exact(cli, ID_BYTES)
            cli.sendall(b"\x01")
            return payload, PeerLinks(rank, [cli])
        except (OSError, RuntimeError) as exc:
            last = exc
            cli.close()
            time.sleep(min(0.1, max(0.0, deadline - time.monotonic())))
    raise RuntimeError(f"Rank {rank} failed to connect to master at {master_addr}") from last


def exchange_id(rank: int, world_size: int, master_addr: str, timeout: float, make_id) -> bytes:
    """rendezvous() without the liveness channel: returns the id bytes."""
    payload, links = rendezvous(rank, world_size, master_addr, timeout, make_id)
    links.close()
    return payload


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(ID_BYTES)
    L.check(L.load().orca_comm_get_unique_id(ctypes.cast(buf, ctypes.c_void_p)))
    return buf.raw


class NcclCommunicator:
    """One NCCL communicator per process/GPU (orca_comm_*)."""

    def __init__(self, backend, rank: int, world_size: int, unique_id: bytes,
                 timeout: float = _DEFAULT_TIMEOUT_SECONDS):
        _validate_process_group(rank, world_size)
        timeout = _validate_timeout(timeout)
        if len(unique_id) != ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        self.backend = backend
        self.rank, self.world_size = rank, world_size
        idbuf = ctypes.create_string_buffer(bytes(unique_id), ID_BYTES)
        h = ctypes.c_void_p()
        L.check(L.load().orca_comm_init(backend.ctx, rank, world_size,
                                        ctypes.cast(idbuf, ctypes.c_void_p), timeout,
                                        ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def allreduce_avg(self, dev_ptr: int, n: int):
        L.check(L.load().orca_comm_allreduce_avg(self._h, ctypes.c_void_p(dev_ptr), int(n)))

    def abort(self):
        if getattr(self, "_h", None):
            L.load().orca_comm_abort(self._h)

    def close(self):
        if getattr(self, "_h", None):
            L.check(L.load().orca_comm_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DistributedDataParallel:
    """DDP wrapper around an MlpTrainer with the reference's constructor
    (module, rank, world_size, master_addr, timeout).  The communicator is set
    up lazily on the first step, like the reference's lazy _connect."""

    def __init__(self, module, rank: int = 0, world_size: int = 1,
                 master_addr: str = "127.0.0.1:18888", timeout: float = _DEFAULT_TIMEOUT_SECONDS,
                 bucket_bytes: int = 0):
        from .mlp import MlpTrainer
        if not isinstance(module, MlpTrainer):
            raise TypeError("module must be an orcaml_b200.mlp.MlpTrainer instance")
        _validate_process_group(rank, world_size)
        self.module = module
        self.rank, self.world_size = rank, world_size
        self.master_addr = master_addr
        self.timeout = _validate_timeout(timeout)
        self.host, self.port = _parse_master_addr(master_addr)
        self.bucket_bytes = int(bucket_bytes)
        self.comm = None
        self.links = None

    def _connect(self):
        if self.comm is not None or self.world_size <= 1:
            return
        uid, self.links = rendezvous(self.rank, self.world_size, self.master_addr, self.timeout,
                                     nccl_unique_id)
        self.comm = NcclCommunicator(self.module.backend, self.rank, self.world_size, uid, self.timeout)
        # A step waits on its peers through the gradient all-reduce; bound that
        # wait by the same timeout the reference applies to its peer sockets.
        self.module.backend.set_timeout(self.timeout)
        self.module.attach_comm(self.comm, self.bucket_bytes)

    def parameters(self):
        return self.module.get_parameters()

    def step(self, x, t) -> float:
        """One data-parallel step.  A peer that stops taking part surfaces as
        RuntimeError, as a lost peer socket does in the reference
        (python/orca/distributed.py:65-80): one that left between steps is
        seen on the rendezvous sockets before anything is launched; one that
        stays but never joins makes the all-reduce miss the `timeout`
        deadline.  The communicator is then aborted and this wrapper cannot
        step again."""
        self._connect()
        try:
            if self.links is not None:
                self.links.check()
            return self.module.step(x, t)
        except (RuntimeError, L.OrcaTimeout, L.OrcaCommError) as exc:
            if self.comm is not None:
                self.comm.abort()
            if isinstance(exc, RuntimeError):
                raise
            raise RuntimeError(f"Rank {self.rank}: distributed peer stopped responding: {exc}") from exc

    def close(self):
        if self.comm is not None:
            self.module.attach_comm(None)
            self.comm.close()
            self.comm = None
        if self.links is not None:
            self.links.close()
            self.links = None
