"""Set up the NVLS (NVSwitch multicast) region of a DeviceCommunicator.

Rank 0 creates the multicast object and exports it as a POSIX file
descriptor. A descriptor is only meaningful inside a process, so it travels
to the other ranks of the box over a Unix socket in the abstract namespace
(``SCM_RIGHTS``), named through the communicator's out-of-band exchange. Each
rank then adds its GPU, and only after every rank did so binds its own
physical backing and maps both views (see ``csrc/cuda/nvls.cpp``).

Every step ends with an exchange of a status byte, so a failure on any rank
(no NVSwitch, no multicast support, a driver error) turns the feature off on
all ranks together instead of leaving some ranks waiting on a collective the
others will never enter. ``NEXAR_NVLS=0`` disables it.
"""
from __future__ import annotations

import os
import socket
import uuid
from typing import Callable, List


def _all_ok(exchange: Callable[[bytes], List[bytes]], ok: bool) -> bool:
    return all(s == b"1" for s in exchange(b"1" if ok else b"0"))


LAST_REASON = ""


def _fail(native, why: str, release: bool = True) -> bool:
    global LAST_REASON
    LAST_REASON = why
    if release:
        native.nvls_release()
    if os.environ.get("NEXAR_NVLS_DEBUG"):
        print(f"nexar_b200: NVLS disabled: {why}", flush=True)
    return False


def setup_nvls(native, rank: int, world: int, exchange: Callable[[bytes], List[bytes]], nbytes: int,
               timeout_s: float = 120.0) -> bool:
    """Create, share, bind and map the multicast region. Collective over all ranks.

    Returns True when active on every rank; otherwise False on every rank and
    ``LAST_REASON`` says why.
    """
    global LAST_REASON
    want = os.environ.get("NEXAR_NVLS", "1") != "0" and world > 1
    supported = False
    why = "disabled (NEXAR_NVLS=0 or a single rank)" if not want else ""
    if want:
        try:
            supported = bool(native.nvls_supported())
            if not supported:
                why = "device reports no multicast / POSIX-fd handle support"
        except Exception as e:  # noqa: BLE001 - any driver error means "not available"
            supported, why = False, f"capability query failed: {e}"
    # One rank per process: a descriptor handoff to oneself (a single process
    # posing as several ranks) has nobody on the other end.
    votes = exchange(f"{int(supported)}:{os.getpid()}".encode())
    pids = {v.split(b":")[1] for v in votes}
    if not all(v.startswith(b"1:") for v in votes):
        return _fail(native, why or "unsupported on a peer rank", release=False)
    if len(pids) != world:
        return _fail(native, "ranks share a process", release=False)
    err = None
    if rank == 0:
        srv = None
        try:
            fd = native.nvls_create(nbytes)
            name = f"nexar-nvls-{os.getpid()}-{uuid.uuid4().hex}"
            srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            srv.bind("\0" + name)
            srv.listen(world)
            srv.settimeout(timeout_s)
        except Exception as e:  # noqa: BLE001
            err, name = e, ""
        names = exchange(name.encode())
        if err is None:
            try:
                for _ in range(world - 1):
                    conn, _ = srv.accept()
                    with conn:
                        socket.send_fds(conn, [b"N"], [fd])
            except Exception as e:  # noqa: BLE001
                err = e
        if srv is not None:
            srv.close()
        del names
    else:
        names = exchange(b"")
        name = names[0].decode()
        if not name:
            err = RuntimeError("rank 0 could not create the multicast object")
        else:
            try:
                s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
                s.settimeout(timeout_s)
                s.connect("\0" + name)
                _, fds, _, _ = socket.recv_fds(s, 1, 1)
                s.close()
                native.nvls_import(fds[0], nbytes)
            except Exception as e:  # noqa: BLE001
                err = e
    if not _all_ok(exchange, err is None):
        return _fail(native, f"multicast object create/share failed: {err}")
    try:
        native.nvls_add_device()
    except Exception as e:  # noqa: BLE001
        err = e
    if not _all_ok(exchange, err is None):  # every device added before anyone binds
        return _fail(native, f"cuMulticastAddDevice failed: {err}")
    try:
        native.nvls_bind_map()
    except Exception as e:  # noqa: BLE001
        err = e
    if not _all_ok(exchange, err is None):
        return _fail(native, f"bind/map failed: {err}")
    LAST_REASON = "active"
    return True
