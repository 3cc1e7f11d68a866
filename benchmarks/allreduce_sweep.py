"""Allreduce size sweep, one rank per GPU under torchrun:

    torchrun --nproc-per-node N benchmarks/allreduce_sweep.py [--graph] [--algos ...] [--reference]

Contiguous bf16 buffers from 4 KB to 256 MB (powers of two plus 10/16/24 MB),
N(0,1) values seeded per rank. Every in-house algorithm (one-shot push,
one-shot pull, two-shot, NVLS when present) and the reference's NCCL path
(torch.distributed.all_reduce), eager and CUDA-graph-captured. With
--reference at TP=2 it also times the reference's own MailboxAR (unmodified
sglang/mailbox_all_reduce.py + mailbox_ar_ext.cu from baseline/_ref, JIT-built
from source; sizes up to its 24 MB limit). Times are CUDA events on the
launching stream, max over ranks; bus bandwidth = 2(n-1)/n * bytes / t
(the reference reports algbw at n=2, tests/mailbox_sweep.py:3, which equals
busbw there). Prints one JSON line per (size, impl, mode).
"""
import argparse
import datetime
import importlib
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"

SIZES = [1 << p for p in range(12, 29)] + [10 << 20, 16 << 20, 24 << 20]


def busbw(nbytes, ms, n):
    return 2 * (n - 1) / n * nbytes / (ms * 1e-3) / 1e9


def timed(fn, iters, group):
    torch.cuda.synchronize()
    dist.barrier(group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def graph_of(fn, reps):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    return g


def load_reference():
    """The unmodified reference communicator (copied as-is into baseline/_ref)."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref", "sglang")
    if not os.path.isfile(os.path.join(ref_dir, "mailbox_all_reduce.py")):
        return None, "baseline/_ref/sglang missing"
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", os.path.join(ROOT, "baseline", "_ref", "torch_extensions"))
    sys.path.insert(0, ref_dir)
    try:
        mod = importlib.import_module("mailbox_all_reduce")
        return mod, None
    except Exception as e:  # noqa: BLE001
        return None, repr(e)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--graph", action="store_true", help="also time CUDA-graph replays")
    ap.add_argument("--graph-replays", type=int, default=1000)
    ap.add_argument("--algos", default="auto,oneshot_push,oneshot_pull,twoshot,twoshot_push,nvls,nccl")
    ap.add_argument("--reference", action="store_true")
    ap.add_argument("--max-bytes", type=int, default=256 << 20)
    ap.add_argument("--out", default=None)
    ap.add_argument("--sizes", default=None, help="comma-separated byte counts (default: the full sweep)")
    ap.add_argument("--norm", action="store_true",
                    help="time the fused allreduce + residual + RMSNorm on [bytes/8192, 4096] bf16 rows "
                         "(one-shot push, two-shot, two-shot push; NCCL + the norm kernel as the baseline) "
                         "instead of the plain allreduce")
    ap.add_argument("--trace", action="store_true",
                    help="also print block 0's phase timestamps (us from kernel start) of the last of 20 "
                         "back-to-back calls, per rank")
    args = ap.parse_args()

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    group = dist.group.WORLD
    comm_mod = importlib.import_module(f"{PKG}.parallel.communicator")
    cfg_mod = importlib.import_module(f"{PKG}.config")
    # explicit algorithms run in-house at every size; "auto" follows the
    # product policy (in-house up to the per-world max_size, NCCL above)
    policy_max = cfg_mod.CommConfig.from_env().max_size_for(world)
    ar = comm_mod.MailboxAR(None, dev, max_size=max(args.max_bytes, 256 << 20))
    assert not ar.disabled
    algos = [a for a in args.algos.split(",") if a]
    if "nvls" in algos and "nvls" not in ar.transport:
        algos.remove("nvls")
    ref = None
    if args.reference and world == 2:
        mod, err = load_reference()
        if mod is not None:
            try:
                mod._SHIM_BYTES = 0  # as its own sweep does (tests/mailbox_sweep.py:23-27)
                ref = mod.MailboxAR(None, local)
                if ref.disabled:
                    ref = None
            except Exception as e:  # noqa: BLE001
                err = repr(e)
                ref = None
        if ref is None and rank == 0:
            print(json.dumps({"impl": "reference_mailbox", "unavailable": err}), flush=True)
        if ref is not None:
            algos.append("reference_mailbox")
    out_f = open(args.out, "a") if (args.out and rank == 0) else None
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    sizes = [int(v) for v in args.sizes.split(",")] if args.sizes else SIZES
    trace = torch.zeros(8, dtype=torch.int64, device=dev)
    for nbytes in sorted(set(s for s in sizes if s <= args.max_bytes)):
        n = nbytes // 2
        x = torch.randn(n, device=dev, generator=g).to(torch.bfloat16)
        o = torch.empty_like(x)
        iters = max(10, min(1000, int(2e9 // nbytes)))
        if args.norm:
            H = 4096
            M = max(1, nbytes // (2 * H))
            xn = x[:M * H].view(M, H)
            resn = torch.zeros(M, H, device=dev, dtype=torch.bfloat16)
            on = torch.empty_like(xn)
            wn = torch.ones(H, device=dev, dtype=torch.bfloat16)
            ops = importlib.import_module(f"{PKG}.ops")
        for algo in algos:
            if args.norm:
                if algo == "nccl":
                    y = xn.clone()

                    def fn():
                        dist.all_reduce(y, group=group)
                        ops.fused_add_rmsnorm(y, resn, wn, 1e-5, out=on)
                elif algo in ("oneshot_push", "twoshot", "twoshot_push"):
                    if M * H * 2 > ar.fused_rmsnorm_limit() or (
                            algo == "oneshot_push" and M * H * 2 > ar._ar.chunk_limit(comm_mod.ALGO_ONESHOT_PUSH)):
                        continue
                    fn = lambda a=comm_mod.ALGO_IDS[algo]: ar.all_reduce_rmsnorm(xn, resn, wn, 1e-5, out=on,  # noqa
                                                                                 algo=a)
                else:
                    continue
            elif algo == "nccl":
                y = x.clone()
                fn = lambda: dist.all_reduce(y, group=group)  # noqa: E731
            elif algo == "reference_mailbox":
                if nbytes > ref.max_size:
                    continue
                fn = lambda: ref.custom_all_reduce(x)  # noqa: E731
            elif algo == "auto" and nbytes > policy_max:
                y = x.clone()
                fn = lambda: dist.all_reduce(y, group=group)  # noqa: E731
            else:
                a = None if algo == "auto" else algo
                fn = lambda a=a: ar.custom_all_reduce(x, algo=a, out=o)  # noqa: E731
            for _ in range(5):
                fn()
            modes = [("eager", None)]
            if args.graph and algo != "reference_mailbox":
                modes.append(("graph", args.graph_replays))
            for mode, reps in modes:
                if mode == "eager":
                    ms = timed(fn, iters, group)
                else:
                    k = 10
                    gr = graph_of(fn, k)
                    ms = timed(gr.replay, max(1, reps // k), group) / k
                    del gr
                rec = {"bytes": nbytes, "impl": algo, "mode": mode, "tp": world, "us": ms * 1e3,
                       "busbw_gbs": busbw(nbytes, ms, world)}
                if args.norm:
                    rec["op"] = "allreduce+residual+rmsnorm"
                    rec["rows"] = M
                if algo == "auto" and not args.norm:
                    rec["route"] = "nccl" if nbytes > policy_max else "mailbox"
                if rank == 0:
                    print(json.dumps(rec), flush=True)
                    if out_f:
                        out_f.write(json.dumps(rec) + "\n")
            if args.trace and algo not in ("nccl", "reference_mailbox") and not (algo == "auto" and nbytes > policy_max):
                trace.zero_()
                ar._ar.set_trace(trace.data_ptr())
                torch.cuda.synchronize()
                dist.barrier(group)
                for _ in range(20):
                    fn()
                torch.cuda.synchronize()
                ar._ar.set_trace(0)
                allm = [None] * world
                dist.all_gather_object(allm, trace.tolist(), group=group)
                if rank == 0:
                    t0 = min(m[0] for m in allm)
                    print(json.dumps({"bytes": nbytes, "impl": algo, "norm": bool(args.norm), "trace_us": [
                        [round((v - t0) / 1e3, 2) if v else None for v in m[:6]] for m in allm]}), flush=True)
        if ar.err():
            raise SystemExit(f"communicator error {ar.status()}")
    dist.barrier()
    ar.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
