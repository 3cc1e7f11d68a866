"""FD exchange over abstract Unix sockets (the transport of cuMem POSIX-FD
handles between ranks), tested with memfds on CPU ranks."""
import os

from _mp import run_ranks


def _exchange(rank, world):
    from importlib import import_module

    bs = import_module("3080_mod_p2p_sglang_patch_b200.parallel.bootstrap")
    fd = os.memfd_create(f"r{rank}")
    os.write(fd, f"rank-{rank}".encode())
    session = bs.session_id()
    got = bs.exchange_fds(session, rank, world, fd, timeout_ms=20000)
    seen = {}
    for p, pfd in got.items():
        os.lseek(pfd, 0, 0)
        seen[p] = os.read(pfd, 64).decode()
        os.close(pfd)
    bfd = bs.broadcast_fd(session, rank, world, fd if rank == 0 else -1, 0, timeout_ms=20000)
    os.lseek(bfd, 0, 0)
    from_root = os.read(bfd, 64).decode()
    if bfd != fd:
        os.close(bfd)
    os.close(fd)
    return seen, from_root


def test_fd_exchange_3_ranks():
    res = run_ranks(_exchange, 3)
    for r, (seen, from_root) in res.items():
        assert seen == {p: f"rank-{p}" for p in range(3) if p != r}
        assert from_root == "rank-0"
