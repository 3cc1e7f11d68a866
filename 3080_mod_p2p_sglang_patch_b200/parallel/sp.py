"""Sequence-parallel (SP) collectives fused into the TP GEMMs.

With SP the residual stream between layers is sharded by token rows: rank r
owns rows [r*Mo, r*Mo + Mo), Mo = ceil(M / world). Around every RMSNorm:

* row-parallel GEMM (o_proj, down_proj) -> reduce-scatter: the tcgen05 GEMM
  epilogue pushes each finished output row to its owner's slot over NVLink
  (``gemm_rs``);
* ``rs_norm_ag``: the owner sums its rows over ranks (rank order, fp32, one
  rounding), adds them to its residual shard, applies RMSNorm and pushes the
  normed rows into every rank's gather buffer G, then raises its flag;
* all-gather -> column-parallel GEMM (QKV, gate_up): ``gemm_ag`` reads A from
  G; its TMA producer waits for the flags of the owners of each 128-row tile
  before loading it, so tiles whose rows have landed start while others are
  still in flight, and no separate all-gather launch exists.

The reference has no sequence parallelism; the B200 build adds it for the
70B serving configuration (reference call stack of the TP allreduce:
sglang/mailbox_all_reduce.py:172-181, which SP replaces by RS + AG).

Buffers live in a dedicated symmetric allocation sized for the engine's
largest chunk (``max_rows`` x ``hidden``), so they never move: every launch
is CUDA-graph safe. No NVLS/multicast mapping is used here.
"""
import logging

import torch

from .._ext import cuda_ext
from ..utils import launches
from .communicator import MailboxError

logger = logging.getLogger(__name__)

MiB = 1 << 20


def _round_up(x, g):
    return (x + g - 1) // g * g


class SequenceParallel:
    """SP buffers and launches of one TP group (collective construction)."""

    def __init__(self, comm, max_rows: int, hidden: int):
        from .symm import SymmetricBuffer, _raw_uint8

        C = cuda_ext()
        self.comm = comm
        self.rank = comm.rank
        self.world = comm.world_size
        self.device = comm.device
        self.max_rows = int(max_rows)
        self.hidden = int(hidden)
        mo = -(-self.max_rows // self.world)
        self.rs_bytes = _round_up(self.world * mo * self.hidden * 2, MiB)
        self.g_bytes = _round_up(self.max_rows * self.hidden * 2, MiB)
        size = C.SIG_BYTES + 2 * self.rs_bytes + self.g_bytes
        self._buf = SymmetricBuffer(size, self.device, comm.group, nvls=False,
                                    timeout_ms=comm.cfg.handshake_timeout_ms)
        self._state = torch.zeros(C.STATE_WORDS, dtype=torch.int32, device=self.device)
        self._status = C.host_mapped_alloc(4 * C.STATUS_WORDS)
        self._ar = C.ArComm(self.rank, self.world, list(self._buf.ptrs), 0, self._state.data_ptr(), self._status.dev,
                            self._status.host, 0, 0, comm.cfg.timeout_ns, self.rs_bytes, self.g_bytes)
        self._gather = _raw_uint8(self._ar.sp_gather_ptr(), self.g_bytes, self.device).view(torch.bfloat16)
        self.max_blocks = comm.cfg.max_blocks
        torch.cuda.synchronize(self.device)
        logger.info("[MailboxAR] sequence parallel ready rank=%d rows=%d hidden=%d (%.0f MiB)", self.rank,
                    self.max_rows, self.hidden, size / MiB)

    # ------------------------------------------------------------------ shapes
    def rows_per_rank(self, M: int) -> int:
        return -(-M // self.world)

    def own_rows(self, M: int):
        """(first row, number of rows) owned by this rank for an M-row batch."""
        mo = self.rows_per_rank(M)
        r0 = min(M, self.rank * mo)
        return r0, max(0, min(M, r0 + mo) - r0)

    def fits(self, M: int, N: int = None) -> bool:
        N = self.hidden if N is None else N
        return M * N * 2 <= self.g_bytes and self.world * self.rows_per_rank(M) * N * 2 <= self.rs_bytes

    # ------------------------------------------------------------------ launches
    def _check(self):
        code = self._ar.error()
        if code:
            st = self._ar.status()
            raise MailboxError(f"[MailboxAR] rank {self.rank}: sequence-parallel wait gave up (code {code}, "
                               f"block {st[1]}, peer {st[2]}, phase {st[3]}, epoch {st[4]})")

    def rs_push(self, x: torch.Tensor):
        """Reduce-scatter a local [M, H] tensor (e.g. the vocab-parallel
        embedding partial): every row goes to its owner's slot."""
        self._check()
        self._ar.sp_rs_push(x, self.max_blocks)
        launches.add(1)

    def gemm_rs(self, a: torch.Tensor, w: torch.Tensor):
        """Row-parallel GEMM a @ w^T whose epilogue pushes every output row to
        its owner (reduce-scatter fused into the GEMM)."""
        from .. import ops

        self._check()
        self._ar.gemm_rs(a, w, ops.workspace(a.device).err)
        launches.add(1)

    def rs_norm_ag(self, M: int, res_own: torch.Tensor, w: torch.Tensor, eps: float):
        """res_own += sum over ranks of the owned rows; G <- rmsnorm(res_own) * w
        on every rank (all-gather pushed by the owners)."""
        self._check()
        self._ar.sp_rs_norm_ag(M, res_own, w, eps, self.max_blocks)
        launches.add(1)

    def gemm_ag(self, M: int, w: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
        """out[M, N] = G[M, H] @ w^T, each 128-row tile loaded once its owners'
        rows of the last ``rs_norm_ag`` have landed."""
        from .. import ops

        C = cuda_ext()
        N, K = w.shape
        if out is None:
            out = torch.empty((M, N), dtype=torch.bfloat16, device=w.device)
        ws = ops.workspace(w.device)
        splits = C.gemm_plan(M, N, K)[1]
        wbuf = ws.gemm(splits * M * N) if splits > 1 else None
        self._check()
        self._ar.sp_gemm_ag(M, w, out, wbuf, ws.err)
        launches.add(2 if splits > 1 else 1)
        return out

    def gathered(self, M: int) -> torch.Tensor:
        """G[:M] after waiting (on the device) for every owner's rows: for
        consumers other than ``gemm_ag`` (e.g. the LM head's last rows)."""
        self._ar.sp_ag_wait(M)
        launches.add(1)
        return self._gather[: M * self.hidden].view(M, self.hidden)

    # ------------------------------------------------------------------ state
    def err(self) -> int:
        return int(self._ar.error()) if self._ar is not None else 0

    def reset(self):
        """Clear flags, epochs and the error word (the owner calls it collectively)."""
        torch.cuda.synchronize(self.device)
        self._buf.zero_signals(cuda_ext().SIG_BYTES)
        self._state.zero_()
        self._ar.clear_status()
        torch.cuda.synchronize(self.device)

    def close(self):
        if self._buf is not None:
            self._gather = None
            self._buf.close()
            self._buf = None
        if self._status is not None:
            cuda_ext().host_mapped_free(self._status.host)
            self._status = None
        self._ar = None
