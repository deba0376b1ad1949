"""Out-of-band hand-over of the communicator id (rank 0 -> all ranks).

This is the only control-plane step of the multi-GPU path: NCCL needs every
rank to hold the same ids (``MMP_COMM_ID_BYTES``) before ``mmp_comm_init``.  Two
transports:

* torch's ``TCPStore`` when torch is importable.  Under ``torchrun`` the
  launcher's agent already serves a store at ``MASTER_ADDR:MASTER_PORT``
  (``TORCHELASTIC_USE_AGENT_STORE=True``) and every rank connects to it as a
  client; otherwise rank 0 hosts the store.  torch is used as a key-value
  store only: no tensor and no process group is created.
* a plain TCP socket otherwise (or with ``MMP_RDZV=socket``): rank 0 listens
  on ``MASTER_ADDR:MASTER_PORT`` (``MASTER_PORT + 1`` under torchrun's agent
  store, or ``MMP_RDZV_PORT``), the other ranks connect and read the bytes.

Both give up after ``timeout_s`` with ``TimeoutError``, so a rank that never
arrives ends the others with an error instead of a hang.
"""

from __future__ import annotations

import os
import socket
import time

__all__ = ["exchange_root_bytes"]

_generation = [0]


def _agent_store() -> bool:
    return os.environ.get("TORCHELASTIC_USE_AGENT_STORE", "").lower() == "true"


def _addr_port() -> tuple[str, int]:
    addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = os.environ.get("MASTER_PORT")
    if not port and not os.environ.get("MMP_RDZV_PORT"):
        raise RuntimeError("MASTER_PORT (or MMP_RDZV_PORT) must be set for a multi-rank communicator")
    return addr, int(port or 0)


def _socket_port(port: int) -> int:
    # under torchrun the launcher's store already listens on MASTER_PORT
    if os.environ.get("MMP_RDZV_PORT"):
        return int(os.environ["MMP_RDZV_PORT"])
    return port + 1 if _agent_store() else port


def transport() -> str:
    """"store" (torch's TCPStore) or "socket".  Deciding imports torch when
    it is present: call this before NCCL is opened, so that a torch in the
    process loads its own NCCL first and the library's dlopen then returns
    that same copy (torch does not import against an older NCCL that is
    already loaded)."""
    if os.environ.get("MMP_RDZV", "") == "socket":
        return "socket"
    try:
        import torch.distributed  # noqa: F401
    except ImportError:
        return "socket"
    return "store"


def _via_store(payload, rank, world, timeout_s, nbytes):
    import datetime

    from torch.distributed import TCPStore  # key-value store only

    addr, port = _addr_port()
    agent = _agent_store()
    kw = {} if agent else {"multi_tenant": True}
    store = TCPStore(addr, port, world, is_master=(rank == 0 and not agent),
                     timeout=datetime.timedelta(seconds=timeout_s), **kw)
    key = "mmp_comm_id/%s/%d" % (os.environ.get("TORCHELASTIC_RESTART_COUNT", "0"), _generation[0])
    if rank == 0:
        store.set(key, bytes(payload))
        got = bytes(payload)
    else:
        got = bytes(store.get(key))  # waits up to the store timeout
    # keep rank 0's store (and its server) alive until every rank has read
    store.add(key + "/read", 1)
    if rank == 0:
        t0 = time.monotonic()
        while int(store.add(key + "/read", 0)) < world:
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError("communicator id: not every rank collected it in time")
            time.sleep(0.002)
    if len(got) != nbytes:
        raise RuntimeError("communicator id has the wrong size")
    return got


def _recv_exact(s, n):
    buf = b""
    while len(buf) < n:
        chunk = s.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("rendezvous peer closed the connection")
        buf += chunk
    return buf


def _via_socket(payload, rank, world, timeout_s, nbytes):
    addr, port = _addr_port()
    port = _socket_port(port)
    deadline = time.monotonic() + timeout_s
    if rank == 0:
        srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        srv.bind((addr, port))
        srv.listen(world)
        try:
            for _ in range(world - 1):
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError("communicator id: a rank did not connect in time")
                srv.settimeout(left)
                try:
                    c, _ = srv.accept()
                except socket.timeout as e:
                    raise TimeoutError("communicator id: a rank did not connect in time") from e
                with c:
                    c.sendall(bytes(payload))
        finally:
            srv.close()
        return bytes(payload)
    while True:
        try:
            s = socket.create_connection((addr, port), timeout=max(deadline - time.monotonic(), 0.1))
            break
        except OSError:
            if time.monotonic() > deadline:
                raise TimeoutError("communicator id: rank 0 did not answer in time")
            time.sleep(0.05)
    with s:
        s.settimeout(max(deadline - time.monotonic(), 0.1))
        return _recv_exact(s, nbytes)


def exchange_root_bytes(payload, rank: int, world: int, timeout_s: float = 120.0, nbytes: int = 128,
                        how: str | None = None) -> bytes:
    """Rank 0 passes ``payload`` (``nbytes`` bytes, or a callable that makes
    them, called on rank 0 after the transport is chosen); every rank
    returns those bytes."""
    how = how or transport()
    if rank == 0 and callable(payload):
        payload = payload()
    if world <= 1:
        return bytes(payload)
    _generation[0] += 1
    if how == "store":
        return _via_store(payload, rank, world, timeout_s, nbytes)
    return _via_socket(payload, rank, world, timeout_s, nbytes)
