"""Helpers to run a function on N gloo ranks (CPU) in child processes."""
import multiprocessing as mp
import os
import traceback


def _entry(fn, rank, world, port, q, args):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        res = fn(rank, world, *args)
        q.put((rank, "ok", res))
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass
    except BaseException:  # noqa: BLE001
        q.put((rank, "err", traceback.format_exc()))


def run_ranks(fn, world, args=(), timeout=240):
    from conftest import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=timeout)
            if status != "ok":
                raise AssertionError(f"rank {rank} failed:\n{payload}")
            results[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results
