"""Launch each hot sm_100a kernel once on a small-but-real case, for ncu.

    python benchmarks/profile_kernels.py [--which gemm,fmha,decode]

Cases (a few hundred MB on the device at most):
  gemm   : tcgen05 GEMM, 8B gate_up at TP=1 (M=1024, N=28672, K=4096)
  fmha   : tcgen05 prefill attention, 1024 queries at context 4096, 32q/8kv heads
  decode : tensor-core decode attention, batch 64, context 4096, 32q/8kv heads
Each kernel runs exactly once (plus nothing else from this package), so
`ncu -k regex:<name> -c 1` captures it.
"""
import argparse
import importlib
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--which", default="gemm,fmha,decode")
    args = ap.parse_args()
    ops = importlib.import_module(f"{PKG}.ops")
    which = args.which.split(",")
    D, P = 128, 16
    if "gemm" in which:
        a = torch.randn(1024, 4096, device="cuda").to(torch.bfloat16)
        w = (torch.randn(28672, 4096, device="cuda") * 0.02).to(torch.bfloat16)
        ops.gemm(a, w)
        torch.cuda.synchronize()
        del a, w
    if "fmha" in which or "decode" in which:
        L = 4096
        nblk = L // P
        kc = torch.randn(nblk * 64, 8, P, D, device="cuda").to(torch.bfloat16)
        vc = torch.randn_like(kc)
    if "fmha" in which:
        q = torch.randn(1024, 32, D, device="cuda").to(torch.bfloat16)
        bt = torch.arange(nblk, dtype=torch.int32, device="cuda").view(1, -1)
        cu = torch.tensor([0, 1024], dtype=torch.int32, device="cuda")
        kvl = torch.tensor([L], dtype=torch.int32, device="cuda")
        ops.prefill_attention(q, kc, vc, cu, kvl, bt, ops.prefill_tiles([1024]).cuda())
        torch.cuda.synchronize()
    if "decode" in which:
        B = 64
        q = torch.randn(B, 32, D, device="cuda").to(torch.bfloat16)
        bt = torch.arange(B * nblk, dtype=torch.int32, device="cuda").view(B, nblk) % kc.shape[0]
        kvl = torch.full((B,), L, dtype=torch.int32, device="cuda")
        ops.decode_attention(q, kc, vc, kvl, bt, splits=1)
        torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    print("profile_kernels done")


if __name__ == "__main__":
    main()
