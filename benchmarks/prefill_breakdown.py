"""Per-kernel device-time breakdown of TP prefill chunks (shares, not a
benchmark number: the times come from the CUDA profiler's kernel records).

    torchrun --nproc-per-node N benchmarks/prefill_breakdown.py [--impl native|torch] [--prompt-len 4096]

One request of --prompt-len tokens is prefilled (chunk 1024, the prefill CUDA
graph for the native build) once to warm up and once under torch.profiler.
Kernel times are summed per category on every rank; rank 0 prints the max
over ranks per category as one JSON line, plus the top kernels.
"""
import argparse
import collections
import importlib
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"

CATEGORIES = [
    ("allreduce", ("ar_", "fused_rs_norm", "fused_allsum", "nccl", "allreduce", "seg_")),
    ("attention", ("fmha", "attention", "attn", "flash")),
    ("gemm", ("gemm", "splitk", "cutlass", "sm100", "sm90", "nvjet", "cublas", "xmma")),
    ("norm", ("rmsnorm",)),
    ("rope_kv", ("rope",)),
    ("silu", ("silu",)),
    ("embed_argmax", ("embedding", "argmax")),
]


def category(name: str) -> str:
    n = name.lower()
    for cat, keys in CATEGORIES:
        if any(k in n for k in keys):
            return cat
    return "other"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", default="native", choices=["native", "torch"])
    ap.add_argument("--model", default="8b")
    ap.add_argument("--prompt-len", type=int, default=4096)
    ap.add_argument("--chunk", type=int, default=1024)
    args = ap.parse_args()
    par = importlib.import_module(f"{PKG}.parallel")
    models = importlib.import_module(f"{PKG}.models")
    eng_mod = importlib.import_module(f"{PKG}.engine")
    rank, world, local = par.init_distributed(timeout_s=300)
    dev = torch.device("cuda", local)
    tp = par.TPGroup(None, dev, use_mailbox=(args.impl == "native")) if world > 1 else None
    cfg = models.LlamaConfig.by_name(args.model)
    eng = eng_mod.LLMEngine(cfg, tp=tp, max_batch=2, max_seq=args.prompt_len + 16, chunk=args.chunk, seed=0,
                            use_graphs=False, impl=args.impl, prefill_graph=(args.impl == "native"))
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, cfg.vocab, (args.prompt_len,), generator=g).tolist()
    eng.generate([prompt], max_new_tokens=1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        eng.generate([prompt], max_new_tokens=1)
        torch.cuda.synchronize()
    per_cat = collections.Counter()
    per_kernel = collections.Counter()
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time_total > 0:
            us = ev.device_time_total
            per_cat[category(ev.name)] += us
            per_kernel[ev.name[:90]] += us
    cats = [c for c, _ in CATEGORIES] + ["other"]
    t = torch.tensor([per_cat[c] for c in cats], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        chunks = -(-args.prompt_len // args.chunk)
        rec = {"impl": args.impl, "tp": world, "model": cfg.name, "prompt_len": args.prompt_len, "chunks": chunks,
               "ms_per_chunk": {c: round(v / 1e3 / chunks, 3) for c, v in zip(cats, t.tolist())},
               "top_kernels_ms_per_chunk": [(k, round(v / 1e3 / chunks, 3)) for k, v in per_kernel.most_common(12)]}
        rec["total_ms_per_chunk"] = round(sum(rec["ms_per_chunk"].values()), 3)
        print(json.dumps(rec), flush=True)
    if tp is not None:
        tp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
