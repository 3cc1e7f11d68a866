"""One GPU standing in for W tensor-parallel ranks (tests, smoke, profiling).

The communicator's kernels meet their peers at cross-rank barriers, so the
ranks' blocks must run at the same time. Separate launches on one GPU give no
such guarantee, so ``EmulatedWorld`` runs every rank's blocks in ONE
cooperative launch (``_C.ar_emulated``: rank = blockIdx.y, the same device
code as the multi-GPU launch). Each emulated rank has its own symmetric buffer
(a plain local allocation), state words and host-mapped status words, and its
``ArComm`` context lists all W buffers as its "peers".

Kernels that wait only on flags set by EARLIER launches (the push epilogue of
the fused GEMM, its push-all reduction, the sequence-parallel pushes) run as
ordinary per-rank launches in rank order on one stream: each wait is already
satisfied when it starts. The device waits are bounded (``timeout_ms``), so a
wrong order reports an error instead of waiting.

The reference tests its protocol only with two real GPUs and two processes
(tests/test_mailbox_torch.py, tests/hammer_mbx.py); this is the one-GPU
counterpart for the kernels that replace it.
"""
import torch

from .._ext import cuda_ext
from .communicator import ALGO_ONESHOT_PUSH, ALGO_TWOSHOT_PUSH, DTYPE_IDS, MailboxError


class EmulatedWorld:
    """W emulated ranks on ``device``.

    ``half_bytes`` / ``fuse_half_bytes``: size of one ping-pong half of the
    allreduce and fused-GEMM regions of every rank's buffer. ``blocks``:
    blocks per rank of every emulated launch (all W x blocks must be
    co-resident: W * blocks <= 148 at 512 threads).
    """

    def __init__(self, world: int, device=None, half_bytes: int = 8 << 20, fuse_half_bytes: int = 8 << 20,
                 timeout_ms: float = 200.0, blocks: int = 8):
        if world < 2 or world > 8:
            raise ValueError("world must be 2..8")
        self.C = C = cuda_ext()
        self.world = world
        self.device = torch.device(device if device is not None else "cuda")
        self.blocks = int(blocks)
        size = C.SIG_BYTES + 2 * half_bytes + 2 * fuse_half_bytes
        self.bufs = [torch.zeros(size, dtype=torch.uint8, device=self.device) for _ in range(world)]
        self.states = [torch.zeros(C.STATE_WORDS, dtype=torch.int32, device=self.device) for _ in range(world)]
        self.status = [C.host_mapped_alloc(4 * C.STATUS_WORDS) for _ in range(world)]
        ptrs = [b.data_ptr() for b in self.bufs]
        self.comms = [
            C.ArComm(r, world, ptrs, 0, self.states[r].data_ptr(), self.status[r].dev, self.status[r].host,
                     half_bytes, 0, int(timeout_ms * 1e6), fuse_half_bytes)
            for r in range(world)
        ]
        self._scratch = torch.zeros(C.EMU_RANK_BYTES * world, dtype=torch.uint8, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ helpers
    def _launch(self, op, algo, dtype, ins, outs, residuals=(), weight=0, nbytes=0, M=0, N=0, eps=0.0, threads=512):
        self.check()
        self.C.ar_emulated(self.comms, op, algo, dtype, [int(p) for p in ins], [int(p) for p in outs],
                           [int(p) for p in residuals], int(weight), int(nbytes), int(M), int(N), float(eps),
                           self.blocks, self._scratch.data_ptr(), self._scratch.numel(), int(threads))

    def check(self):
        """Raise MailboxError if any emulated rank recorded a device error."""
        for r, c in enumerate(self.comms):
            code = c.error()
            if code:
                st = c.status()
                raise MailboxError(f"emulated rank {r}: device error {code} (block {st[1]}, peer {st[2]}, "
                                   f"phase {st[3]}, epoch {st[4]})")

    def epochs(self):
        """Allreduce epoch of every emulated rank (device words)."""
        return [int(s[0].item()) for s in self.states]

    # ------------------------------------------------------------------ collectives
    def allreduce(self, xs, algo=ALGO_ONESHOT_PUSH, outs=None):
        """outs[r] = sum over ranks of xs (one emulated launch); ``outs=xs``
        reduces in place."""
        if outs is None:
            outs = [torch.empty_like(x) for x in xs]
        nbytes = xs[0].numel() * xs[0].element_size()
        self._launch(self.C.EMU_ALLREDUCE, algo, DTYPE_IDS[xs[0].dtype], [x.data_ptr() for x in xs],
                     [o.data_ptr() for o in outs], nbytes=nbytes)
        return outs

    def all_reduce_rmsnorm(self, xs, residuals, weight, eps, algo=ALGO_TWOSHOT_PUSH, threads=512):
        """residuals[r] += sum(xs); outs[r] = rmsnorm(residuals[r]) * weight.
        ``threads=256``: the half-size blocks of overlapped micro-batches."""
        M, N = xs[0].shape
        outs = [torch.empty_like(x) for x in xs]
        self._launch(self.C.EMU_AR_RMSNORM, algo, DTYPE_IDS[torch.bfloat16], [x.data_ptr() for x in xs],
                     [o.data_ptr() for o in outs], [r.data_ptr() for r in residuals], weight.data_ptr(),
                     nbytes=M * N * 2, M=M, N=N, eps=eps, threads=threads)
        return outs

    def all_gather(self, xs):
        """outs[r][k] = xs[k] for every rank r."""
        outs = [torch.empty((self.world,) + tuple(x.shape), dtype=x.dtype, device=x.device) for x in xs]
        nbytes = xs[0].numel() * xs[0].element_size()
        self._launch(self.C.EMU_ALLGATHER, ALGO_ONESHOT_PUSH, DTYPE_IDS[torch.bfloat16], [x.data_ptr() for x in xs],
                     [o.data_ptr() for o in outs], nbytes=nbytes)
        return outs

    def gemm_all_reduce_rmsnorm(self, a_s, w_s, residuals, norm_w, eps, push_all=True):
        """The fused row-parallel GEMM -> allreduce -> residual + RMSNorm of
        every rank: each rank's GEMM epilogue pushes its partial tiles (rank
        order, one launch per rank), then the reductions run (push-all: one
        launch per rank, each waiting only on the finished GEMMs' flags;
        owner-push: one emulated launch, its reduce and all-gather meet at a
        barrier)."""
        M, N = a_s[0].shape[0], w_s[0].shape[0]
        outs = [torch.empty((M, N), dtype=torch.bfloat16, device=self.device) for _ in range(self.world)]
        self.check()
        for r in range(self.world):
            self.comms[r].gemm_push(a_s[r], w_s[r], self.err, bool(push_all))
        if push_all:
            for r in range(self.world):
                self.comms[r].fused_allsum_norm(M, N, residuals[r].data_ptr(), norm_w.data_ptr(), outs[r].data_ptr(),
                                                float(eps), self.blocks)
        else:
            self._launch(self.C.EMU_FUSED_RS_NORM, 0, DTYPE_IDS[torch.bfloat16], [0] * self.world,
                         [o.data_ptr() for o in outs], [r.data_ptr() for r in residuals], norm_w.data_ptr(),
                         M=M, N=N, eps=eps)
        return outs

    def close(self):
        torch.cuda.synchronize(self.device)
        for s in self.status:
            self.C.host_mapped_free(s.host)
        self.status = []
        self.comms = []
        self.bufs = []

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
        return False
