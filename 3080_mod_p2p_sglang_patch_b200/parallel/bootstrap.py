"""Host-side rendezvous helpers for the communicator.

Object collectives go through the communicator's process group (gloo or
NCCL), as the reference's handle exchange does
(sglang/mailbox_all_reduce.py:116,127,138). File descriptors (cuMem / NVLS
handles) cannot travel through pickles, so they go over abstract Unix sockets
with SCM_RIGHTS (native code in csrc/cpu/fdx.cpp); the socket names embed a
session id that rank 0 draws and everyone learns through the group.
"""
import os
import uuid

import torch.distributed as dist

from .._ext import cpu_ext


def all_gather_obj(obj, group=None):
    world = dist.get_world_size(group=group)
    out = [None] * world
    dist.all_gather_object(out, obj, group=group)
    return out


def agree(ok: bool, group=None) -> bool:
    """True only if every rank passed ``ok=True`` (consistent decision)."""
    return all(bool(x) for x in all_gather_obj(bool(ok), group))


def session_id(group=None) -> str:
    """A short id drawn by the group's first rank, known to every rank."""
    mine = f"{os.getpid()}-{uuid.uuid4().hex[:12]}"
    return all_gather_obj(mine, group)[0]


def sock_name(session: str, rank: int, what: str) -> str:
    return f"mbx-{session}-{what}-{rank}"


def exchange_fds(session: str, rank: int, world: int, my_fd: int, group=None, timeout_ms: int = 60000, what="mem"):
    """Send ``my_fd`` to every other rank and receive theirs.

    Returns ``{peer_rank: fd}`` (fds owned by the caller). Every rank must call
    this with the same ``session``/``what``. Raises on failure after taking part
    in every collective step (the lockstep rule of the reference,
    sglang/mailbox_all_reduce.py:83-89).
    """
    ext = cpu_ext()
    lfd = -1
    err = None
    try:
        lfd = ext.fdx_listen(sock_name(session, rank, what))
    except Exception as e:  # noqa: BLE001 - reported through the consensus
        err = e
    ok = agree(err is None, group)  # everybody listening before anyone sends
    if not ok:
        if lfd >= 0:
            ext.fdx_close(lfd)
        raise RuntimeError(f"fd exchange: listen failed on some rank ({err})")
    got = {}
    try:
        for p in range(world):
            if p != rank:
                ext.fdx_send(sock_name(session, p, what), rank, [my_fd], timeout_ms)
        for tag, fds in ext.fdx_recv(lfd, world - 1, timeout_ms):
            got[int(tag)] = fds[0]
    except Exception as e:  # noqa: BLE001
        err = e
    finally:
        ext.fdx_close(lfd)
    ok = agree(err is None and len(got) == world - 1, group)
    if not ok:
        for fd in got.values():
            os.close(fd)
        raise RuntimeError(f"fd exchange failed on some rank ({err})")
    return got


def broadcast_fd(session: str, rank: int, world: int, fd: int, src: int = 0, group=None, timeout_ms=60000,
                 what="mc"):
    """Rank ``src`` sends ``fd`` to everyone; returns the received fd (or ``fd`` on ``src``)."""
    ext = cpu_ext()
    lfd = -1
    err = None
    if rank != src:
        try:
            lfd = ext.fdx_listen(sock_name(session, rank, what))
        except Exception as e:  # noqa: BLE001
            err = e
    if not agree(err is None, group):
        if lfd >= 0:
            ext.fdx_close(lfd)
        raise RuntimeError(f"fd broadcast: listen failed ({err})")
    out = fd
    try:
        if rank == src:
            for p in range(world):
                if p != src:
                    ext.fdx_send(sock_name(session, p, what), src, [fd], timeout_ms)
        else:
            (tag, fds), = ext.fdx_recv(lfd, 1, timeout_ms)
            out = fds[0]
    except Exception as e:  # noqa: BLE001
        err = e
    finally:
        if lfd >= 0:
            ext.fdx_close(lfd)
    if not agree(err is None, group):
        raise RuntimeError(f"fd broadcast failed ({err})")
    return out
