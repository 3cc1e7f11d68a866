"""MailboxAR: a CustomAllreduce-shaped tensor-parallel allreduce communicator.

Public surface kept from the reference (sglang/mailbox_all_reduce.py:62-225):
``MailboxAR(group, device, max_size)``, ``.disabled``, ``.should_custom_ar``,
``.custom_all_reduce``, ``.capture``, ``.register_graph_buffers``, ``.close``,
the segmented-overlap API ``.get_seg_stream`` / ``.submit_seg`` /
``.wait_seg`` / ``.seg_err``, and the ``[MailboxAR] ready rank=.. attempt=..
mbx=.. peer=..`` log line.

What is different on B200:

* world sizes 2..8 (the reference is TP=2 only, :69-71);
* buffers are cuMem symmetric memory mapped once over NVLink 5 (plus an NVLS
  multicast mapping when present) instead of a driver-patched BAR1 window;
* one kernel launch per allreduce, algorithm by size and world size:
  one-shot push (the mailbox data path), two-shot, NVLS multimem;
* messages larger than one buffer half are chunked in-house up to
  ``max_size``; above it (or for unsupported dtypes/layouts)
  ``should_custom_ar`` is False and the caller uses NCCL, like the reference;
* the device error word is host-mapped and checked on every call: a timed-out
  wait raises ``MailboxError`` instead of silently returning garbage (the
  reference's sticky, unchecked ``err``, mailbox_ar_ext.cu:26-50);
* on CPU tensors (gloo groups) the same protocol runs in the native CPU
  mailbox engine over shared memory.
"""
import contextlib
import logging
import os

import torch
import torch.distributed as dist

from .._ext import cpu_ext, cuda_ext
from ..config import CommConfig
from ..utils import launches
from . import bootstrap, faults

logger = logging.getLogger(__name__)

# dtype ids shared with the kernels (reference numbering, mailbox_ar_ext.cu:123)
DTYPE_IDS = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

ALGO_AUTO, ALGO_ONESHOT_PUSH, ALGO_ONESHOT_PULL, ALGO_TWOSHOT, ALGO_NVLS, ALGO_TWOSHOT_PUSH = 0, 1, 2, 3, 4, 5
ALGO_NAMES = {ALGO_ONESHOT_PUSH: "oneshot_push", ALGO_ONESHOT_PULL: "oneshot_pull", ALGO_TWOSHOT: "twoshot",
              ALGO_NVLS: "nvls", ALGO_TWOSHOT_PUSH: "twoshot_push"}
ALGO_IDS = {v: k for k, v in ALGO_NAMES.items()}

ERROR_NAMES = {3: "barrier/flag wait timed out", 4: "segment wait timed out", 5: "segment slot-free wait timed out",
               6: "fused-epilogue wait timed out"}


class MailboxError(RuntimeError):
    """A device-side wait of the communicator gave up (peer missing or late)."""


def is_weak_contiguous(inp: torch.Tensor) -> bool:
    """Contiguous, or a view whose storage tail from the offset is exactly its
    elements (the sglang/vLLM notion the reference imports, :46-52)."""
    return inp.is_contiguous() or (
        inp.storage().nbytes() - inp.storage_offset() * inp.element_size() == inp.numel() * inp.element_size()
    )


class MailboxAR:
    """Tensor-parallel allreduce over NVLink symmetric memory.

    ``group``: process group of the TP ranks (``None`` = default group).
    ``device``: CUDA device (int or torch.device) for the GPU transport, or
    ``"cpu"`` for the shared-memory CPU transport.
    ``max_size``: largest message (bytes) handled here; larger ones go to NCCL.
    """

    def __init__(self, group=None, device=None, max_size=None, config: CommConfig = None):
        self.disabled = True
        self.group = group
        self.cfg = config or CommConfig.from_env()
        self.rank = dist.get_rank(group=group)
        self.world_size = dist.get_world_size(group=group)
        self.max_size = int(max_size if max_size is not None else self.cfg.max_size_for(self.world_size))
        self.counters = {**{name: 0 for name in ALGO_NAMES.values()}, "cpu": 0, "fallback": 0, "errors": 0, "fused": 0,
                         "allgather": 0}
        self._buf = None
        self._ar = None
        self._cpu = None
        self._status = None
        self._seg_seq = 0
        self._seg_stream = None
        self.sp = None
        self.mbx = 0
        self.peer_mbx = 0
        if self.world_size < 2 or self.world_size > 8:
            logger.info("[MailboxAR] world size %d not in 2..8, using NCCL", self.world_size)
            return
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        if isinstance(device, int):
            device = torch.device("cuda", device)
        if isinstance(device, str):
            device = torch.device(device)
        self.device = device
        ok = False
        attempt = -1
        for attempt in range(2):
            err = None
            faults.set_attempt(attempt)
            try:
                if device.type == "cuda":
                    self._setup_gpu()
                else:
                    self._setup_cpu()
            except Exception as e:  # noqa: BLE001 - decision made collectively below
                err = e
                logger.warning("[MailboxAR] attempt %d failed: %s", attempt, e)
                self._teardown()
            # every rank takes part in every consensus step (lockstep rule)
            if bootstrap.agree(err is None, group):
                ok = True
                break
            self._teardown()
        if not ok:
            logger.error("[MailboxAR] setup failed on some rank; falling back to NCCL on every rank")
            return
        self.disabled = False
        self._attempt = attempt
        logger.info("[MailboxAR] ready rank=%d attempt=%d mbx=%#x peer=%#x", self.rank, attempt, self.mbx,
                    self.peer_mbx)

    # ------------------------------------------------------------------ setup
    def _lane_bytes(self):
        C = cuda_ext()
        return C.SIG_BYTES + 2 * self.cfg.lane_half_bytes if self.cfg.lane_half_bytes else 0

    def _buffer_bytes(self):
        C = cuda_ext()
        seg = C.SEG_SLOTS * C.MAX_RANKS * self.cfg.seg_slot_bytes
        return C.SIG_BYTES + 2 * self.cfg.half_bytes + 2 * self.cfg.fuse_half_bytes + seg + self._lane_bytes()

    def _setup_gpu(self):
        from .symm import SymmetricBuffer

        C = cuda_ext()
        torch.cuda.set_device(self.device)
        self._buf = SymmetricBuffer(self._buffer_bytes(), self.device, self.group, nvls=self.cfg.nvls,
                                    timeout_ms=self.cfg.handshake_timeout_ms)
        self._state = torch.zeros(C.STATE_WORDS, dtype=torch.int32, device=self.device)
        self._status = C.host_mapped_alloc(4 * C.STATUS_WORDS)
        self._ar = C.ArComm(self.rank, self.world_size, list(self._buf.ptrs), int(self._buf.mc_ptr),
                            self._state.data_ptr(), self._status.dev, self._status.host, self.cfg.half_bytes,
                            self.cfg.seg_slot_bytes, self.cfg.timeout_ns, self.cfg.fuse_half_bytes)
        torch.cuda.synchronize(self.device)
        self.mbx = self._buf.local_ptr
        self.peer_mbx = self._buf.ptrs[(self.rank + 1) % self.world_size]
        self.transport = self._buf.transport + ("+nvls" if self._buf.mc_ptr else "")
        # the second lane's region ends the buffer (after the segment slots)
        self._lane_off = self._buffer_bytes() - self._lane_bytes()
        self._lane = None

    def _setup_cpu(self):
        ext = cpu_ext()
        session = bootstrap.session_id(self.group)
        path = f"/dev/shm/mbx-{session}"
        err = None
        if self.rank == 0:
            try:
                faults.check("cpu_open", self.rank)
                self._cpu = ext.CpuMailbox(path, self.rank, self.world_size, self.cfg.cpu_slot_bytes, True,
                                           self.cfg.cpu_timeout_ms)
            except Exception as e:  # noqa: BLE001
                err = e
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"CPU mailbox creation failed ({err})")
        if self.rank != 0:
            try:
                faults.check("cpu_open", self.rank)
                self._cpu = ext.CpuMailbox(path, self.rank, self.world_size, self.cfg.cpu_slot_bytes, False,
                                           self.cfg.cpu_timeout_ms)
            except Exception as e:  # noqa: BLE001
                err = e
        # everyone mapped before rank 0 may unlink the file on close
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"CPU mailbox open failed ({err})")
        self.transport = "cpu-shm"
        self.mbx = 0
        self.peer_mbx = 0

    def _teardown(self):
        lane = getattr(self, "_lane", None)
        if lane is not None:
            lane.release()
            self._lane = None
        if self.sp is not None:
            try:
                self.sp.close()
            except Exception:  # noqa: BLE001
                pass
            self.sp = None
        if self._buf is not None:
            try:
                self._buf.close()
            except Exception:  # noqa: BLE001
                pass
            self._buf = None
        if self._status is not None:
            try:
                cuda_ext().host_mapped_free(self._status.host)
            except Exception:  # noqa: BLE001
                pass
            self._status = None
        if self._cpu is not None:
            self._cpu.close()
            self._cpu = None
        self._ar = None

    # ------------------------------------------------------------------ gating
    def should_custom_ar(self, inp: torch.Tensor) -> bool:
        """Same gate as the reference (:160-170): dtype, 16-byte size, weak
        contiguity, size limit, plus the tensor being on this transport's device."""
        if self.disabled:
            return False
        if inp.dtype not in DTYPE_IDS:
            return False
        nbytes = inp.numel() * inp.element_size()
        if nbytes % 16 != 0:
            return False
        if not is_weak_contiguous(inp):
            return False
        if self._cpu is not None:
            if inp.device.type != "cpu" or nbytes > self._cpu.slot_bytes():
                return False
        elif inp.device != self.device:
            return False
        return nbytes <= self.max_size

    def pick_algo(self, nbytes: int) -> int:
        """Algorithm by size and world size (tuned thresholds in CommConfig)."""
        if nbytes <= self.cfg.oneshot_max.get(self.world_size, 0):
            return ALGO_ONESHOT_PUSH
        if self._buf is not None and self._buf.mc_ptr and nbytes >= self.cfg.nvls_min and \
                self.world_size >= self.cfg.nvls_min_world:
            return ALGO_NVLS
        return ALGO_TWOSHOT_PUSH

    # ------------------------------------------------------------------ calls
    def _check_error(self):
        if self._ar is not None:
            code = self._ar.error()
            if code:
                self.counters["errors"] += 1
                st = self._ar.status()
                raise MailboxError(
                    f"[MailboxAR] rank {self.rank}: {ERROR_NAMES.get(code, 'error')} (code {code}, block {st[1]}, "
                    f"peer {st[2]}, phase {st[3]}, epoch {st[4]}); call reset() on every rank or fall back to NCCL")

    def custom_all_reduce(self, input: torch.Tensor, algo=None, out: torch.Tensor = None):
        """Out-of-place allreduce (sum). Returns None when gated off (the caller
        then uses NCCL), like the reference (:172-181)."""
        if self.disabled or not self.should_custom_ar(input):
            return None
        if out is None:
            out = torch.empty_like(input)
        self._all_reduce_into(input, out, algo)
        return out

    def all_reduce(self, input: torch.Tensor, out: torch.Tensor = None, algo=None, inplace: bool = False):
        """Allreduce that always succeeds: in-house when gated on, NCCL/gloo otherwise."""
        if self.should_custom_ar(input):
            if inplace:
                out = input
            elif out is None:
                out = torch.empty_like(input)
            self._all_reduce_into(input, out, algo)
            return out
        self.counters["fallback"] += 1
        t = input if inplace else input.clone()
        dist.all_reduce(t, group=self.group)
        if out is not None and out is not t:
            out.copy_(t)
            return out
        return t

    def _all_reduce_into(self, input, out, algo):
        nbytes = input.numel() * input.element_size()
        if self._cpu is not None:
            inp = input.contiguous()
            code = self._cpu.allreduce(inp.data_ptr(), out.data_ptr(), nbytes, DTYPE_IDS[input.dtype])
            self.counters["cpu"] += 1
            if code:
                self.counters["errors"] += 1
                raise MailboxError(f"[MailboxAR] rank {self.rank}: CPU mailbox wait timed out (code {code}, "
                                   f"peer {self._cpu.error_peer()})")
            return out
        self._check_error()
        if isinstance(algo, str):
            algo = ALGO_IDS[algo]
        a = algo or self.pick_algo(nbytes)
        if a == ALGO_NVLS and not self._buf.mc_ptr:
            a = ALGO_TWOSHOT
        self._ar.allreduce(input.data_ptr(), out.data_ptr(), nbytes, DTYPE_IDS[input.dtype], a, self.cfg.max_blocks,
                           torch.cuda.current_stream(self.device).cuda_stream)
        self.counters[ALGO_NAMES[a]] += 1
        launches.add(max(1, -(-nbytes // int(self._ar.chunk_limit(a)))))
        return out

    def all_reduce_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                           out: torch.Tensor = None, algo=None, threads: int = 512, max_blocks: int = None):
        """Fused: residual <- bf16(residual + allreduce(x)); returns
        rmsnorm(residual) * weight (bf16), in one kernel launch.

        ``threads=256`` launches half-size blocks (half the registers per
        block), so each fits on an SM beside a running GEMM CTA: the form
        used when the call overlaps compute on another stream; ``max_blocks``
        caps the grid below the configured one for the same reason."""
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and residual.is_contiguous()
        H = x.shape[-1]
        M = x.numel() // H
        nbytes = x.numel() * 2
        if out is None:
            out = torch.empty_like(x)
        self._check_error()
        if algo is None:
            algo = ALGO_ONESHOT_PUSH if nbytes <= self.cfg.oneshot_max.get(self.world_size, 0) else ALGO_TWOSHOT_PUSH
        self._ar.ar_rmsnorm(x.data_ptr(), residual.data_ptr(), weight.data_ptr(), out.data_ptr(), M, H, eps, algo,
                            int(max_blocks or self.cfg.max_blocks), torch.cuda.current_stream(self.device).cuda_stream,
                            int(threads))
        self.counters["fused"] += 1
        launches.add(1)
        return out

    def fused_push_all(self, M: int, N: int) -> bool:
        """Push every row to every rank (one exchange) for 2 ranks; push rows to
        their owner (reduce-scatter + all-gather, less traffic) beyond."""
        return self.world_size <= 2

    def fused_gemm_fits(self, M: int, N: int) -> bool:
        """Whether an [M, N] bf16 output fits the fused GEMM->allreduce buffer."""
        if self._ar is None or N % 8:
            return False
        W = self.world_size
        if self.fused_push_all(M, N):
            need = W * M * N * 2
        else:
            Mo = -(-M // W)
            need = W * Mo * N * 2 + M * N * 2
        return need <= self._ar.fused_capacity()

    def gemm_all_reduce_rmsnorm(self, a: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                                norm_w: torch.Tensor, eps: float, out: torch.Tensor = None, push_all: bool = None):
        """Row-parallel GEMM fused with the allreduce: the GEMM epilogue stores
        its partial output tiles straight into the owner ranks' symmetric
        buffers (reduce-scatter overlapped with the remaining tiles), then one
        launch reduces the owned rows, all-gathers them and applies
        residual <- residual + sum, out = rmsnorm(residual) * norm_w."""
        from .. import ops

        M, N = a.shape[0], w.shape[0]
        if out is None:
            out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
        self._check_error()
        if push_all is None:
            push_all = self.fused_push_all(M, N)
        self._ar.gemm_ar_rmsnorm(a, w, residual, norm_w, out, eps, ops.workspace(a.device).err, self.cfg.max_blocks,
                                 bool(push_all))
        self.counters["fused"] += 1
        launches.add(2)
        return out

    def fused_rmsnorm_limit(self) -> int:
        """Largest message (bytes) the fused allreduce+RMSNorm takes in one launch."""
        if self._ar is None:
            return 0
        # two-shot push needs W row slots plus the reduced rows in one half
        return int(self.cfg.half_bytes // 2 - 16 * self.world_size * 8192)

    def all_gather(self, x: torch.Tensor, out: torch.Tensor = None):
        """out[r] = x of rank r (shape [world, *x.shape]), one launch."""
        if out is None:
            out = torch.empty((self.world_size,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        self._check_error()
        self._ar.allgather(x.data_ptr(), out.data_ptr(), x.numel() * x.element_size(), self.cfg.max_blocks,
                           torch.cuda.current_stream(self.device).cuda_stream)
        self.counters["allgather"] += 1
        launches.add(1)
        return out

    # ------------------------------------------------------------------ second lane
    def lane(self):
        """A second communication context for collectives issued from another
        stream, concurrently with this one's (``None`` without the GPU
        transport or with ``lane_half_bytes = 0``).

        It lives in a disjoint region at the end of the same symmetric
        buffers, with its own signal words, ping-pong halves, device epochs and
        host-mapped status, so its calls and the main context's may run at
        the same time and in either order; the calls of each context must
        still come in the same order on every rank. Creating it is local (the
        memory is mapped already)."""
        if self._ar is None or not self.cfg.lane_half_bytes:
            return None
        if self._lane is None:
            self._lane = _Lane(self)
        return self._lane

    # ------------------------------------------------------------------ graph
    def capture(self):
        """Graph capture needs nothing: every kernel argument is a fixed
        address and the epochs live on the device (reference :183-185)."""
        return contextlib.nullcontext()

    def register_graph_buffers(self):
        """No-op: the symmetric buffers never move (reference :218-219)."""

    # ------------------------------------------------------------------ segmented overlap
    def get_seg_stream(self):
        if self._seg_stream is None:
            self._seg_stream = torch.cuda.Stream(device=self.device)
        return self._seg_stream

    @property
    def seg_slot_capacity(self) -> int:
        return self.cfg.seg_slot_bytes

    def submit_seg(self, input: torch.Tensor, stream=None) -> int:
        """Push one segment to every peer's slot on ``stream`` (side stream).
        The device keeps the sequence number (graph-replay safe); the returned
        host counter mirrors it for API parity with the reference (:194-203)."""
        assert not self.disabled and self._ar is not None
        stream = stream or self.get_seg_stream()
        self._seg_seq += 1
        self._ar.seg_submit(input.data_ptr(), input.numel() * input.element_size(), self.cfg.max_blocks,
                            stream.cuda_stream)
        return self._seg_seq

    def wait_seg(self, seq: int, local_seg: torch.Tensor, out_seg: torch.Tensor) -> None:
        """On the current stream: wait for every peer's segment ``seq``, then
        out = sum over ranks (own part from ``local_seg``). Segments must be
        waited in submission order."""
        self._ar.seg_wait(local_seg.data_ptr(), out_seg.data_ptr(), local_seg.numel() * local_seg.element_size(),
                          DTYPE_IDS[local_seg.dtype], self.cfg.max_blocks,
                          torch.cuda.current_stream(self.device).cuda_stream)

    def seg_err(self) -> int:
        return self.err()

    # ------------------------------------------------------------------ status
    def sp_setup(self, max_rows: int, hidden: int):
        """Collective: allocate the sequence-parallel buffers for batches of up
        to ``max_rows`` tokens of width ``hidden`` (see parallel/sp.py).
        Returns the ``SequenceParallel`` object (also ``self.sp``), or None on
        the CPU transport or when the communicator is off."""
        if self.disabled or self._ar is None:
            return None
        if self.sp is not None and self.sp.max_rows >= max_rows and self.sp.hidden == hidden:
            return self.sp
        from .sp import SequenceParallel

        if self.sp is not None:
            torch.cuda.synchronize(self.device)
            bootstrap.agree(True, self.group)
            self.sp.close()
        self.sp = SequenceParallel(self, max_rows, hidden)
        return self.sp

    def err(self) -> int:
        """Sticky device error code (0 = ok), read from host-mapped memory."""
        if self._ar is not None:
            code = int(self._ar.error())
            if code == 0 and self.sp is not None:
                code = self.sp.err()
            if code == 0 and self._lane is not None:
                code = self._lane.err()
            return code
        if self._cpu is not None:
            return int(self._cpu.error())
        return 0

    def status(self) -> dict:
        st = self._ar.status() if self._ar is not None else [self.err(), 0, 0, 0, 0]
        return {"err": st[0], "block": st[1], "peer": st[2], "phase": st[3], "epoch": st[4],
                "transport": getattr(self, "transport", None), "counters": dict(self.counters)}

    def epoch(self) -> int:
        """Device epoch (number of completed in-house allreduce launches)."""
        if self._cpu is not None:
            return int(self._cpu.epoch())
        return int(self._state[0].item())

    def reset(self):
        """Collective: clear epochs, flags and the error word on every rank."""
        if self.disabled:
            return
        bootstrap.agree(True, self.group)
        if self._cpu is not None:
            self._cpu.reset()
        else:
            torch.cuda.synchronize(self.device)
            self._buf.zero_signals(cuda_ext().SIG_BYTES)
            self._state.zero_()
            self._ar.clear_status()
            torch.cuda.synchronize(self.device)
            if self.sp is not None:
                self.sp.reset()
            if self._lane is not None:
                self._lane.reset()
        self._seg_seq = 0
        bootstrap.agree(True, self.group)

    def debug_set_epoch(self, epoch: int):
        """Collective, tests only: put every rank at allreduce epoch ``epoch``
        with every barrier flag at the same value (the state after that many
        calls), e.g. just below 2^32 to run the bounded waits across the wrap."""
        if self.disabled:
            return
        bootstrap.agree(True, self.group)
        e = int(epoch) & 0xFFFFFFFF
        if self._cpu is not None:
            self._cpu.set_epoch(e)
        else:
            from .symm import _raw_uint8

            C = cuda_ext()
            signed = e - (1 << 32) if e >= (1 << 31) else e
            torch.cuda.synchronize(self.device)
            _raw_uint8(self._buf.local_ptr, 4 * C.BAR_WORDS, self.device).view(torch.int32).fill_(signed)
            self._state[0] = signed
            torch.cuda.synchronize(self.device)
        bootstrap.agree(True, self.group)

    def check_health(self) -> bool:
        """Collective: True if no rank has an error; otherwise every rank
        disables the communicator (consistent NCCL fallback)."""
        ok = bootstrap.agree(self.err() == 0, self.group)
        if not ok:
            logger.error("[MailboxAR] error on some rank; disabling on every rank (NCCL fallback)")
            self.disabled = True
        return ok

    def close(self):
        """Collective when the GPU transport is up: every rank finishes its
        in-flight launches and passes a barrier before any mapping is released
        (the reference leaves its IPC handles open, mailbox_all_reduce.py:221)."""
        if self._buf is not None or self._cpu is not None:
            if self._buf is not None:
                torch.cuda.synchronize(self.device)
            try:
                bootstrap.agree(True, self.group)
            except Exception:  # noqa: BLE001 - group already gone: release locally
                pass
        self.disabled = True
        self._teardown()

    def __del__(self):
        try:
            self.disabled = True
        except Exception:  # noqa: BLE001
            pass


class _Lane:
    """The second context of a ``MailboxAR`` (see ``MailboxAR.lane``)."""

    def __init__(self, owner: MailboxAR):
        from .symm import _raw_uint8

        C = cuda_ext()
        self.owner = owner
        self.cfg = owner.cfg
        self.device = owner.device
        off = owner._lane_off
        self._sig = _raw_uint8(owner._buf.local_ptr + off, C.SIG_BYTES, owner.device)
        self._state = torch.zeros(C.STATE_WORDS, dtype=torch.int32, device=owner.device)
        self._status = C.host_mapped_alloc(4 * C.STATUS_WORDS)
        ptrs = [p + off for p in owner._buf.ptrs]
        self._ar = C.ArComm(owner.rank, owner.world_size, ptrs, 0, self._state.data_ptr(), self._status.dev,
                            self._status.host, self.cfg.lane_half_bytes, 0, self.cfg.timeout_ns, 0)
        torch.cuda.synchronize(owner.device)

    def err(self) -> int:
        return int(self._ar.error()) if self._ar is not None else 0

    def fits_rmsnorm(self, nbytes: int) -> bool:
        return nbytes <= self.cfg.lane_half_bytes // 2 - 16 * self.owner.world_size * 8192

    def all_reduce_rmsnorm(self, x, residual, weight, eps, out=None, threads: int = 256):
        """Same as ``MailboxAR.all_reduce_rmsnorm`` on this lane, with the
        lane's grid cap (``lane_max_blocks``)."""
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and residual.is_contiguous()
        code = self.err()
        if code:
            raise MailboxError(f"[MailboxAR] rank {self.owner.rank}: second lane: "
                               f"{ERROR_NAMES.get(code, 'error')} (code {code}, status {self._ar.status()})")
        H = x.shape[-1]
        M = x.numel() // H
        nbytes = x.numel() * 2
        if out is None:
            out = torch.empty_like(x)
        algo = ALGO_ONESHOT_PUSH if nbytes <= min(self.cfg.oneshot_max.get(self.owner.world_size, 0),
                                                  int(self._ar.chunk_limit(ALGO_ONESHOT_PUSH))) \
            else ALGO_TWOSHOT_PUSH
        self._ar.ar_rmsnorm(x.data_ptr(), residual.data_ptr(), weight.data_ptr(), out.data_ptr(), M, H, eps, algo,
                            self.cfg.lane_max_blocks, torch.cuda.current_stream(self.device).cuda_stream,
                            int(threads))
        self.owner.counters["fused"] += 1
        launches.add(1)
        return out

    def reset(self):
        """Part of the owner's collective ``reset``: clear this lane's signals,
        epochs and status."""
        torch.cuda.synchronize(self.device)
        self._sig.zero_()
        self._state.zero_()
        self._ar.clear_status()
        torch.cuda.synchronize(self.device)

    def release(self):
        if self._status is not None:
            try:
                cuda_ext().host_mapped_free(self._status.host)
            except Exception:  # noqa: BLE001
                pass
            self._status = None
        self._ar = None
