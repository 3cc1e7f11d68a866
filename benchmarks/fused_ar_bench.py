"""Row-parallel linear + allreduce + residual + RMSNorm at TP = world size:
the fused tcgen05 GEMM -> push-reduce-scatter -> reduce/all-gather/norm pair
vs the same kernels unfused vs two overlapped micro-batches (second half's
GEMM under the first half's collective) vs cuBLAS + NCCL (+ the same norm
kernel).

    torchrun --nproc-per-node N benchmarks/fused_ar_bench.py [--model 8b] [--rows 1024,64,8,1]

CUDA events over --iters back-to-back calls, max over ranks. Reports us per
call and the roofline of the fused pair: max(FLOPs / measured bf16 peak,
bytes over NVLink / 770 GB/s per direction).
"""
import argparse
import datetime
import importlib
import json
import os
import sys

import torch
import torch.distributed as dist
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"
NVLINK_GBS = 770.0


def peak_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)["bf16_tflops"]
    except (OSError, KeyError, ValueError):
        return 1590.0


def timed(fn, iters):
    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) * 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="8b")
    ap.add_argument("--rows", default="1024,64,8,1", help="token counts M")
    ap.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    ops = importlib.import_module(f"{PKG}.ops")
    comm_mod = importlib.import_module(f"{PKG}.parallel.communicator")
    cfg = importlib.import_module(f"{PKG}.models").LlamaConfig.by_name(args.model)
    ar = comm_mod.MailboxAR(None, dev)
    H = cfg.hidden
    shapes = {"o_proj": cfg.heads * cfg.head_dim // world, "down_proj": cfg.ffn // world}
    pk = peak_tflops()
    for name, K in shapes.items():
        w = (torch.randn(H, K, device=dev) * 0.02).to(torch.bfloat16)
        nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
        for M in [int(x) for x in args.rows.split(",")]:
            a = torch.randn(M, K, device=dev).to(torch.bfloat16)
            res = torch.zeros(M, H, device=dev, dtype=torch.bfloat16)
            out = torch.empty(M, H, device=dev, dtype=torch.bfloat16)
            fits = ar.fused_gemm_fits(M, H)

            def fused():
                ar.gemm_all_reduce_rmsnorm(a, w, res, nw, 1e-5, out=out)

            def unfused():
                p = ops.gemm(a, w)
                ar.all_reduce_rmsnorm(p, res, nw, 1e-5, out=out)

            # two micro-batches: the second half's GEMM runs while the first
            # half's allreduce + norm runs on a high-priority side stream
            # (the model's overlapped prefill, reduced to one layer)
            h = (M // 2) // 128 * 128
            comm_s = torch.cuda.Stream(device=dev, priority=-1)
            parts = torch.empty(M, H, device=dev, dtype=torch.bfloat16)
            evs = [torch.cuda.Event() for _ in range(4)]

            def overlapped():
                comp = torch.cuda.current_stream()
                for i, (r0, r1) in enumerate(((0, h), (h, M))):
                    ops.gemm(a[r0:r1], w, out=parts[r0:r1])
                    evs[i].record(comp)
                    with torch.cuda.stream(comm_s):
                        comm_s.wait_event(evs[i])
                        ar.all_reduce_rmsnorm(parts[r0:r1], res[r0:r1], nw, 1e-5, out=out[r0:r1], threads=256)
                        evs[2 + i].record(comm_s)
                comp.wait_event(evs[2])
                comp.wait_event(evs[3])

            def cublas_nccl():
                p = F.linear(a, w)
                dist.all_reduce(p)
                ops.fused_add_rmsnorm(p, res, nw, 1e-5, out=out)

            rec = {"model": cfg.name, "tp": world, "gemm": name, "M": M, "N": H, "K": K}
            if fits:
                rec["fused_us"] = timed(fused, args.iters)
            rec["unfused_us"] = timed(unfused, args.iters)
            if h >= 128:
                rec["overlapped_halves_us"] = timed(overlapped, args.iters)
            rec["cublas_nccl_us"] = timed(cublas_nccl, args.iters)
            flops = 2.0 * M * H * K
            link_bytes = 2.0 * (world - 1) / world * M * H * 2  # reduce-scatter + all-gather, per direction
            roof_us = max(flops / (pk * 1e12), link_bytes / (NVLINK_GBS * 1e9)) * 1e6
            rec["roofline_us"] = roof_us
            if fits:
                rec["fused_frac_of_roofline"] = roof_us / rec["fused_us"]
            if rank == 0:
                print(json.dumps(rec), flush=True)
    assert ar.err() == 0, ar.status()
    dist.barrier()
    ar.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
