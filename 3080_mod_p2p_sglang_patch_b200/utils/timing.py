"""Device timing: CUDA events on the launching stream, bracketed by a barrier
and a synchronize on both sides; multi-GPU numbers are the max over ranks
(the reference times on the host, tests/mailbox_sweep.py:37-53)."""
import torch
import torch.distributed as dist


def max_over_ranks(value: float, group=None) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return value
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def barrier(group=None):
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.barrier(group=group)


class DeviceTimer:
    """with DeviceTimer() as t: ...  ->  t.ms (this rank), t.max_ms (max over ranks)."""

    def __init__(self, group=None, sync_ranks=True):
        self.group = group
        self.sync_ranks = sync_ranks
        self.ms = None
        self.max_ms = None

    def __enter__(self):
        if self.sync_ranks:
            barrier(self.group)
        torch.cuda.synchronize()
        self.e0 = torch.cuda.Event(enable_timing=True)
        self.e1 = torch.cuda.Event(enable_timing=True)
        self.e0.record()
        return self

    def __exit__(self, *exc):
        self.e1.record()
        torch.cuda.synchronize()
        if self.sync_ranks:
            barrier(self.group)
        self.ms = self.e0.elapsed_time(self.e1)
        self.max_ms = max_over_ranks(self.ms, self.group) if self.sync_ranks else self.ms
        return False


def time_fn(fn, iters=10, warmup=3, flush_bytes=0, spacer_cycles=200_000):
    """Per-iteration device ms of fn() (events per iteration, optional L2 flush
    between iterations, excluded from the timing). Returns sorted list.

    A spin kernel of ``spacer_cycles`` runs between the flush and the start
    event, so the host has queued fn()'s kernels before the start event fires:
    otherwise the host's own launch time can fall inside the timed region of
    a kernel shorter than it (the model runs such kernels from CUDA graphs,
    where it does not)."""
    flush = torch.empty(flush_bytes // 4, dtype=torch.float32, device="cuda") if flush_bytes else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        if spacer_cycles:
            torch.cuda._sleep(int(spacer_cycles))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1))
    return sorted(out)
