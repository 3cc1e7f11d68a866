"""Launch each hot sm_100a kernel once on a small-but-real case, for ncu.

    python benchmarks/profile_kernels.py [--which gemm,qkv,fmha,decode]

Cases (a few hundred MB on the device at most):
  gemm   : tcgen05 GEMM, 8B gate_up at TP=1 (M=1024, N=28672, K=4096)
  qkv    : the 8B qkv projection at TP=1, M=1024 N=6144 K=4096 (CTA-pair kernel)
  qkv8   : the 8B qkv shard at TP=8, M=1024 N=768 K=4096 (split-K + reduce), run
           4 times after a 256 MB L2 flush each (capture with -s 3 -c 1 or 2)
  fmha   : tcgen05 prefill attention, 1024 queries at context 4096, 32q/8kv heads
  decode : tensor-core decode attention, batch 64, context 4096, 32q/8kv heads
  fused  : fused row-parallel GEMM -> allreduce -> residual + RMSNorm (push-all
           epilogue + sum/norm launch), then the one-shot allreduce+RMSNorm,
           8B o_proj shape (M=1024, N=4096, K=4096)
  sp     : sequence-parallel GEMM -> reduce-scatter epilogue, owned-row
           RMSNorm + all-gather push, all-gather -> GEMM (same shape)
  elem   : RMSNorm [32768, 4096] and SiLU-mul [8192, 2 x 14336] (inputs > L2)
  int4   : AWQ int4 GEMV, 8 rows, 8B gate_up at TP=1 (N=28672, K=4096, group
           128: 59 MB of packed weights), then its bf16 dequantization
  rope   : q/k-norm RoPE + paged cache write, 8192 tokens, 32q/8kv heads
The fused and sp cases run the multi-GPU kernels as a one-rank emulation
(world = 1): the communicator context points at one local buffer laid out
like the symmetric buffer, so every peer store lands in local memory. They
show the kernels' tensor-core and memory behaviour; NVLink time is not in
them. Each kernel runs exactly once (plus nothing else from this package),
so `ncu -k regex:<name> -c 1` captures it.
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
    if "qkv" in which:
        # the 8B qkv projection at TP=1: a 256 x 192 CTA-pair tile by wave cost
        a = torch.randn(1024, 4096, device="cuda").to(torch.bfloat16)
        w = (torch.randn(6144, 4096, device="cuda") * 0.02).to(torch.bfloat16)
        ops.gemm(a, w)
        torch.cuda.synchronize()
        del a, w
    if "qkv8" in which:
        a = torch.randn(1024, 4096, device="cuda").to(torch.bfloat16)
        w = (torch.randn(768, 4096, device="cuda") * 0.02).to(torch.bfloat16)
        out = torch.empty(1024, 768, device="cuda", dtype=torch.bfloat16)
        flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
        for _ in range(4):
            flush.zero_()
            ops.gemm(a, w, out=out)
        torch.cuda.synchronize()
        del a, w, out, flush
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
    if "fused" in which or "sp" in which:
        C = importlib.import_module(f"{PKG}._ext").cuda_ext()
        M, N, K = 1024, 4096, 4096
        half, fuse_half, g_bytes = 16 << 20, 16 << 20, M * N * 2
        size = C.SIG_BYTES + 2 * half + 2 * fuse_half + g_bytes
        buf = torch.zeros(size, dtype=torch.uint8, device="cuda")
        state = torch.zeros(C.STATE_WORDS, dtype=torch.int32, device="cuda")
        status = C.host_mapped_alloc(4 * C.STATUS_WORDS)
        ar = C.ArComm(0, 1, [buf.data_ptr()], 0, state.data_ptr(), status.dev, status.host, half, 0,
                      2_000_000_000, fuse_half, g_bytes)
        err = ops.workspace("cuda").err
        a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
        res = torch.randn(M, N, device="cuda").to(torch.bfloat16)
        nw = torch.ones(N, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        stream = torch.cuda.current_stream().cuda_stream
        if "fused" in which:
            ar.gemm_ar_rmsnorm(a, w, res, nw, out, 1e-5, err, 148, True)
            part = ops.gemm(a, w)
            ar.ar_rmsnorm(part.data_ptr(), res.data_ptr(), nw.data_ptr(), out.data_ptr(), M, N, 1e-5, 1, 148, stream)
            torch.cuda.synchronize()
        if "sp" in which:
            res_own = res.clone()
            ar.gemm_rs(a, w, err)
            ar.sp_rs_norm_ag(M, res_own, nw, 1e-5, 148)
            ar.sp_gemm_ag(M, w, out, None, err)
            torch.cuda.synchronize()
        assert ar.error() == 0, ar.status()
        C.host_mapped_free(status.host)
    if "elem" in which:
        x = torch.randn(32768, 4096, device="cuda").to(torch.bfloat16)
        nw = torch.ones(4096, device="cuda", dtype=torch.bfloat16)
        ops.rmsnorm(x, nw, 1e-5)
        del x
        gu = torch.randn(8192, 2 * 14336, device="cuda").to(torch.bfloat16)
        ops.silu_mul(gu)
        torch.cuda.synchronize()
        del gu
    if "int4" in which:
        models = importlib.import_module(f"{PKG}.models")
        N, K, G = 28672, 4096, 128
        qw, qz, sc = models.awq_quantize(torch.randn(N, K, device="cuda") * 0.02, G)
        w4 = ops.Int4Weight(qw, qz, sc, G)
        x = torch.randn(8, K, device="cuda").to(torch.bfloat16)
        ops.awq_gemm(x, w4)
        ops.awq_dequant(w4)
        torch.cuda.synchronize()
        del w4, qw, qz, sc
    if "rope" in which:
        T, nq, nkv, page = 8192, 32, 8, 16
        qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda").to(torch.bfloat16)
        cs = ops.rope_cos_sin(T, D, 1e6, "cuda")
        pos = torch.arange(T, dtype=torch.int32, device="cuda")
        kc = torch.zeros(T // page, nkv, page, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        slots = torch.arange(T, dtype=torch.int64, device="cuda")
        nw = torch.ones(D, device="cuda", dtype=torch.bfloat16)
        ops.rope_and_cache(qkv, pos, cs, nq, nkv, slots, kc, vc, q_norm=nw, k_norm=nw, eps=1e-6)
        torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    print("profile_kernels done")


if __name__ == "__main__":
    main()
