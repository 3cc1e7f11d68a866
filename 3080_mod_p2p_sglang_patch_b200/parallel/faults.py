"""Host-side fault injection for the communicator's setup handshakes.

``MBX_INJECT_FAULT="stage@rank[#attempt],..."`` makes ``check(stage, rank)``
raise ``InjectedFault`` on the named rank, at every setup attempt or only at
the given one. Stages are the local operations of the handshakes whose
failure the other ranks learn about only through the all-rank consensus:

  cpu_open     mapping the shared CPU mailbox (CPU transport)
  symm_create  cuMemCreate of the local symmetric buffer
  symm_import  importing a peer's buffer from its POSIX FD
  mc_import    joining the NVLS multicast object (ranks > 0)
  ipc_open     opening a peer's legacy CUDA IPC handle

Tests use it to check that one rank's failure leads every rank to the same
outcome (a retry, the IPC fallback, NVLS off, or NCCL) without a hang. It
only raises on the host: nothing is injected on the GPU. (The reference has
no fault injection; its 16-attempt window-landing retry is the path this
exercises, sglang/mailbox_all_reduce.py:91-146.)
"""
import os

_attempt = 0


class InjectedFault(RuntimeError):
    pass


def set_attempt(attempt: int):
    """The communicator's current setup attempt (0-based)."""
    global _attempt
    _attempt = int(attempt)


def _rules():
    spec = os.environ.get("MBX_INJECT_FAULT", "").strip()
    rules = []
    for item in filter(None, (x.strip() for x in spec.split(","))):
        stage, _, rest = item.partition("@")
        rank, _, att = rest.partition("#")
        rules.append((stage, int(rank), int(att) if att else None))
    return rules


def check(stage: str, rank: int):
    """Raise InjectedFault if a rule names this stage, rank and attempt."""
    for s, r, a in _rules():
        if s == stage and r == rank and (a is None or a == _attempt):
            raise InjectedFault(f"injected fault: {stage} on rank {rank} (attempt {_attempt})")
