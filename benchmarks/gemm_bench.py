"""tcgen05 GEMM vs cuBLAS (torch.matmul) on the model's GEMM shapes.

    python benchmarks/gemm_bench.py [--tp 1,2,4,8] [--m 1024,64,8,1] [--model 8b]

CUDA-event timing per call after warm-up, L2 flushed between calls (a 256 MB
write), median of --iters. Reports TFLOP/s and the fraction of the measured
cuBLAS bf16 peak in MEASURED_PEAKS.json.
"""
import argparse
import importlib
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"


def peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def shapes(cfg, tp):
    H, D = cfg.hidden, cfg.head_dim
    return {
        "qkv": ((cfg.heads + 2 * cfg.kv_heads) // tp * D, H),
        "o": (H, cfg.heads // tp * D),
        "gate_up": (2 * cfg.ffn // tp, H),
        "down": (H, cfg.ffn // tp),
        "lm_head": (cfg.vocab // tp, H),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", default="1,2,8")
    ap.add_argument("--m", default="1024,64,8,1")
    ap.add_argument("--model", default="8b")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    ops = importlib.import_module(f"{PKG}.ops")
    models = importlib.import_module(f"{PKG}.models")
    timing = importlib.import_module(f"{PKG}.utils.timing")
    C = importlib.import_module(f"{PKG}._ext").cuda_ext()
    cfg = models.LlamaConfig.by_name(args.model)
    pk, pk_src = peak()
    flush = 256 << 20
    for tp in [int(x) for x in args.tp.split(",")]:
        for name, (N, K) in shapes(cfg, tp).items():
            w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
            for M in [int(x) for x in args.m.split(",")]:
                if name == "lm_head" and M > 64:
                    continue
                a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
                out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                ours = timing.time_fn(lambda: ops.gemm(a, w, out=out), iters=args.iters, warmup=3, flush_bytes=flush)
                cub = timing.time_fn(lambda: torch.matmul(a, w.t(), out=out), iters=args.iters, warmup=3,
                                     flush_bytes=flush)
                t_o, t_c = ours[len(ours) // 2], cub[len(cub) // 2]
                fl = 2.0 * M * N * K
                bn, splits = C.gemm_plan(M, N, K)
                rec = {"tp": tp, "gemm": name, "M": M, "N": N, "K": K, "bn": bn, "splits": splits,
                       "ours_us": t_o * 1e3, "cublas_us": t_c * 1e3,
                       "ours_tflops": fl / (t_o * 1e-3) / 1e12, "cublas_tflops": fl / (t_c * 1e-3) / 1e12,
                       "ours_frac_of_peak": fl / (t_o * 1e-3) / 1e12 / pk, "peak_src": pk_src,
                       "weight_gbs_ours": N * K * 2 / (t_o * 1e-3) / 1e9, "speedup_vs_cublas": t_c / t_o}
                print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
