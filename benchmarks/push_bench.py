"""NVLink transport bandwidth: the B200 counterpart of the reference's raw
mailbox push bench and CE push bench (sglang/mailbox_ar_ext.cu:201-231,
tests/gate8_ce_bench.py), swept over the number of CTAs.

    torchrun --nproc-per-node N benchmarks/push_bench.py [--mb 64] [--grids 8,16,32,64,148,296]

Every rank moves --mb MB at the same time (so every link carries traffic
both ways, as in an allreduce):

  sm_push1 / sm_push4  SM stores into the next rank's symmetric buffer (1 or 4 16-byte vectors in flight per thread)
  sm_pull4             SM loads from the previous rank's buffer
  ce_push              cudaMemcpyAsync into the next rank's buffer (copy engine)
  nvls_reduce          multimem.ld_reduce (bf16, fp32 accumulate) of this rank's region through the multicast address
  nvls_reduce_noacc    the same without fp32 accumulation
  nvls_store           multimem.st of this rank's region through the multicast address

CUDA events over --iters back-to-back launches, max over ranks; prints one
JSON line per (kind, grid) with GB/s of payload per rank.

--overlap (the reference's tests/gate8_ce_bench.py): the tcgen05 GEMM of
its down_proj shape ([1024, 17408] x [17408, 5120]) alone, a peer push of
the GEMM's output size alone (copy engine, or 16 CTAs of SM stores), the two
serially, and the push on a side stream concurrent with the GEMM; reports
the GEMM slowdown and the time the overlap saves.
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

KINDS = {"sm_push1": 0, "sm_push4": 1, "sm_pull4": 2, "nvls_reduce": 3, "nvls_reduce_noacc": 4, "nvls_store": 5}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mb", type=int, default=64)
    ap.add_argument("--grids", default="8,16,32,64,96,148,296")
    ap.add_argument("--threads", type=int, default=512)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--kinds", default="sm_push1,sm_push4,sm_pull4,ce_push,nvls_reduce,nvls_reduce_noacc,nvls_store")
    ap.add_argument("--overlap", action="store_true", help="GEMM / peer push overlap microbench only")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    C = importlib.import_module(f"{PKG}._ext").cuda_ext()
    symm = importlib.import_module(f"{PKG}.parallel.symm")
    S = args.mb << 20
    buf = symm.SymmetricBuffer(world * S, dev, None, nvls=True)
    src = torch.randn(S // 2, device=dev).to(torch.bfloat16)
    dst = torch.empty_like(src)
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    stream = torch.cuda.current_stream(dev).cuda_stream

    def run(kind, grid):
        if kind == "ce_push":
            return lambda: C.ce_push(buf.ptrs[nxt] + rank * S, src.data_ptr(), S, stream)
        k = KINDS[kind]
        if kind.startswith("sm_push"):
            d, s_ = buf.ptrs[nxt] + rank * S, src.data_ptr()
        elif kind == "sm_pull4":
            d, s_ = dst.data_ptr(), buf.ptrs[prv] + prv * S
        elif kind == "nvls_store":
            d, s_ = buf.mc_ptr + rank * S, src.data_ptr()
        else:
            d, s_ = dst.data_ptr(), buf.mc_ptr + rank * S
        return lambda: C.raw_transport(k, d, s_, S, grid, args.threads, stream)

    if args.overlap:
        overlap(args, C, buf, rank, nxt, dev)
        torch.cuda.synchronize()
        dist.barrier()
        buf.close()
        dist.destroy_process_group()
        return
    grids = [int(g) for g in args.grids.split(",")]
    for kind in args.kinds.split(","):
        if kind.startswith("nvls") and not buf.mc_ptr:
            if rank == 0:
                print(json.dumps({"kind": kind, "unavailable": "no multicast object on this box"}), flush=True)
            continue
        for grid in ([0] if kind == "ce_push" else grids):
            fn = run(kind, grid)
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / args.iters], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item()) * 1e3
            if rank == 0:
                print(json.dumps({"kind": kind, "tp": world, "grid": grid, "threads": args.threads, "bytes": S,
                                  "us": us, "gbs": S / us / 1e3}), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    buf.close()
    dist.destroy_process_group()


def overlap(args, C, buf, rank, nxt, dev):
    ops = importlib.import_module(f"{PKG}.ops")
    M, K, N = 1024, 17408, 5120
    a = torch.randn(M, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    prev = torch.randn(M, N, device=dev).to(torch.bfloat16)  # the tile pushed while the next GEMM runs
    nbytes = prev.numel() * 2
    dst = buf.ptrs[nxt] + rank * nbytes
    assert 2 * nbytes <= buf.size, "buffer too small"
    side = torch.cuda.Stream(device=dev)
    main = torch.cuda.current_stream(dev)

    def gemm():
        ops.gemm(a, w, out=y)

    def push(kind, stream):
        if kind == "ce":
            C.ce_push(dst, prev.data_ptr(), nbytes, stream.cuda_stream)
        else:
            C.raw_transport(KINDS["sm_push4"], dst, prev.data_ptr(), nbytes, 16, 512, stream.cuda_stream)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(main)
        for _ in range(args.iters):
            fn()
        e1.record(main)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.iters * 1e3], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def concurrent(kind):
        side.wait_stream(main)
        push(kind, side)
        gemm()
        main.wait_stream(side)

    g = timed(gemm)
    for kind in ("ce", "sm16"):
        p_ = timed(lambda: push(kind, main))
        serial = timed(lambda: (gemm(), push(kind, main)))
        conc = timed(lambda: concurrent(kind))
        if rank == 0:
            print(json.dumps({"bench": "overlap", "push": kind, "tp": dist.get_world_size(), "gemm_us": g,
                              "push_us": p_, "push_bytes": nbytes, "serial_us": serial, "concurrent_us": conc,
                              "gemm_slowdown": conc / g, "overlap_saved_us": serial - conc}), flush=True)


if __name__ == "__main__":
    main()
