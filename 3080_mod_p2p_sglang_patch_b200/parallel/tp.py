"""Tensor-parallel group state and the allreduce dispatch used by the model.

Plays the role of sglang's GroupCoordinator for the TP group
(``tensor_model_parallel_all_reduce`` -> ``ca_comm.should_custom_ar`` ->
``custom_all_reduce`` or NCCL, the call stack of the reference's hot path).
"""
import datetime
import logging
import os

import torch
import torch.distributed as dist

from ..config import CommConfig, mailbox_enabled
from .communicator import MailboxAR

logger = logging.getLogger(__name__)


class TPGroup:
    """The TP process group plus its communicators.

    ``use_mailbox``: None = follow ``SGLANG_MAILBOX_AR``; True/False force it.
    With one rank every collective is the identity.
    """

    def __init__(self, group=None, device=None, use_mailbox=None, config: CommConfig = None):
        self.group = group
        self.initialized = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if self.initialized else 0
        self.world_size = dist.get_world_size(group) if self.initialized else 1
        self.device = device
        self.ca_comm = None
        # Fused row-parallel GEMM -> allreduce: MBX_FUSED_GEMM_AR=1 forces it on,
        # =0 off; by default on for two ranks, where the epilogue pushes every
        # tile straight to both ranks (one exchange) and measured no slower than
        # GEMM + fused allreduce/norm. With more ranks the owner-push variant
        # needs a reduce-scatter then an all-gather and measured slower.
        env = os.environ.get("MBX_FUSED_GEMM_AR")
        self.fused_gemm_ar = (env == "1") if env in ("0", "1") else self.world_size == 2
        if use_mailbox is None:
            use_mailbox = mailbox_enabled()
        if self.world_size > 1 and use_mailbox:
            self.ca_comm = MailboxAR(group, device, config=config)
            if self.ca_comm.disabled:
                self.ca_comm = None
            else:
                logger.info("[AR] Using MailboxAR (NVLink symmetric-memory mode)")

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world_size == 1:
            return x
        if self.ca_comm is not None:
            out = self.ca_comm.custom_all_reduce(x)
            if out is not None:
                return out
        dist.all_reduce(x, group=self.group)
        return x

    def all_reduce_rmsnorm(self, x, residual, weight, eps, out=None, threads: int = 512):
        """residual += allreduce(x); return rmsnorm(residual) * weight.
        ``threads=256``: the half-size blocks that co-reside with a GEMM
        (calls overlapped with compute on another stream)."""
        from .. import ops

        if self.world_size > 1 and self.ca_comm is not None and self.ca_comm.should_custom_ar(x) and \
                x.numel() * 2 <= self.ca_comm.fused_rmsnorm_limit():
            return self.ca_comm.all_reduce_rmsnorm(x, residual, weight, eps, out=out, threads=threads)
        x = self.all_reduce(x)
        return ops.fused_add_rmsnorm(x, residual, weight, eps, out=out)

    def gemm_all_reduce_rmsnorm(self, a, w, residual, norm_w, eps, out=None):
        """Row-parallel linear + allreduce + residual add + RMSNorm: the fused
        GEMM->collective kernel pair when the communicator is up and the
        output fits its buffer, else GEMM then the fused allreduce+norm."""
        from .. import ops

        M, N = a.shape[0], w.shape[0]
        ca = self.ca_comm
        if self.world_size > 1 and ca is not None and not ca.disabled and M > 64 and self.fused_gemm_ar \
                and ca.fused_gemm_fits(M, N):
            return ca.gemm_all_reduce_rmsnorm(a, w, residual, norm_w, eps, out=out)
        part = ops.gemm(a, w)
        return self.all_reduce_rmsnorm(part, residual, norm_w, eps, out=out)

    def sp_setup(self, max_rows: int, hidden: int):
        """Collective: sequence-parallel buffers on the communicator (None
        without one; see parallel/sp.py)."""
        if self.world_size == 1 or self.ca_comm is None:
            return None
        return self.ca_comm.sp_setup(max_rows, hidden)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """[world, *x.shape]."""
        if self.world_size == 1:
            return x.unsqueeze(0)
        nbytes = x.numel() * x.element_size()
        ca = self.ca_comm
        if ca is not None and ca._ar is not None and nbytes % 16 == 0 and x.is_contiguous() and \
                nbytes <= ca._ar.chunk_limit(1):
            return ca.all_gather(x)
        out = torch.empty((self.world_size,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def close(self):
        if self.ca_comm is not None:
            self.ca_comm.close()
            self.ca_comm = None


def init_distributed(backend: str = None, timeout_s: float = 120.0):
    """Initialise torch.distributed from the torchrun environment (one process
    per GPU). Returns (rank, world_size, local_rank)."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size(), int(os.environ.get("LOCAL_RANK", dist.get_rank()))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1:
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl" and torch.cuda.is_available():
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local
