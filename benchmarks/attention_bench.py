"""Prefill (chunked, causal, paged) and decode (split-KV, paged) attention
throughput on the model's head layout.

    python benchmarks/attention_bench.py [--nq 32 --nkv 8]

Prefill: one 1024-token chunk at context offsets 0/1024/2048/3072 (the
config-3 schedule). Decode: batch {1,8,32,64} at context 4096. CUDA events,
median of iterations; FLOPs count causal work only.
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--nq", type=int, default=32)
    ap.add_argument("--nkv", type=int, default=8)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    ops = importlib.import_module(f"{PKG}.ops")
    timing = importlib.import_module(f"{PKG}.utils.timing")
    D, P = 128, 16
    nq, nkv = args.nq, args.nkv
    L = 4096
    nblk = L // P
    kc = torch.randn(nblk * 64, nkv, P, D, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    for off in (0, 1024, 2048, 3072):
        q_len = 1024
        kv = off + q_len
        q = torch.randn(q_len, nq, D, device="cuda").to(torch.bfloat16)
        bt = torch.arange(nblk, dtype=torch.int32, device="cuda").view(1, -1)
        cu = torch.tensor([0, q_len], dtype=torch.int32, device="cuda")
        kvl = torch.tensor([kv], dtype=torch.int32, device="cuda")
        tiles = ops.prefill_tiles([q_len]).cuda()
        tiles64 = ops.prefill_tiles([q_len], bq=64).cuda()
        flops = 4.0 * D * nq * (q_len * off + q_len * (q_len + 1) / 2)
        sp = ops.prefill_splits(tiles.shape[0], nq, kv)
        for name, fn in (("tcgen05", lambda: ops.prefill_attention(q, kc, vc, cu, kvl, bt, tiles, splits=sp)),
                         ("mma_sync", lambda: ops.prefill_attention_mma(q, kc, vc, cu, kvl, bt, tiles64))):
            t = timing.time_fn(fn, iters=args.iters)
            ms = t[len(t) // 2]
            print(json.dumps({"kind": "prefill", "kernel": name, "q": q_len, "ctx": kv, "nq": nq, "nkv": nkv,
                              "us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12}), flush=True)
    for B in (1, 8, 32, 64):
        q = torch.randn(B, nq, D, device="cuda").to(torch.bfloat16)
        bt = torch.arange(B * nblk, dtype=torch.int32, device="cuda").view(B, nblk) % kc.shape[0]
        kvl = torch.full((B,), L, dtype=torch.int32, device="cuda")
        sp = ops.decode_splits(B, nkv, L)
        t = timing.time_fn(lambda: ops.decode_attention(q, kc, vc, kvl, bt, splits=sp), iters=args.iters,
                           flush_bytes=256 << 20)
        ms = t[len(t) // 2]
        kv_bytes = B * L * nkv * D * 2 * 2
        print(json.dumps({"kind": "decode", "B": B, "ctx": L, "nq": nq, "nkv": nkv, "splits": sp, "us": ms * 1e3,
                          "kv_gbs": kv_bytes / (ms * 1e-3) / 1e9}), flush=True)


if __name__ == "__main__":
    main()
