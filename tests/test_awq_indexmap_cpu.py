"""The int4 kernels' index arithmetic (csrc/quant/awq.cu), restated loop for
loop in numpy: the GEMV's grid / thread / group / 8-row load batches and the
dequantizer's shared-memory tile transpose, on shapes with ragged edges. The
GEMV matches the dense product to fp32 rounding; the dequantizer writes every
element exactly once with the exact value. (Numerics of the compiled kernels
are checked on the GPU in test_ops_gpu.py.)"""
import importlib

import numpy as np
import torch

models = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models")
loader = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models.loader")
ORDER = (0, 2, 4, 6, 1, 3, 5, 7)   # column held by nibble i of a packed word


def unpack8(w):
    w = int(w) & 0xFFFFFFFF
    v = [0.0] * 8
    for i, col in enumerate(ORDER):
        v[col] = float((w >> (4 * i)) & 0xF)
    return np.array(v, np.float32)


def gemv_like_the_kernel(x, qw, qz, sc, G, threads=64):
    M, K = x.shape
    Nq = qw.shape[1]
    N = Nq * 8
    ws = np.zeros((K // G, M, N), np.float32)
    for g in range(K // G):                                   # blockIdx.y
        xs = x[:, g * G:(g + 1) * G].astype(np.float32)
        sumx = xs.sum(1)
        for bx in range((Nq + threads - 1) // threads):       # blockIdx.x
            for t in range(threads):
                c = bx * threads + t
                if c >= Nq:
                    continue
                acc = np.zeros((M, 8), np.float32)
                for k in range(0, G, 8):                      # 8 loads in flight
                    words = [qw[g * G + k + u, c] for u in range(8)]
                    for u in range(8):
                        acc += xs[:, k + u][:, None] * unpack8(words[u])[None, :]
                z = unpack8(qz[g, c])
                s = sc[g, 8 * c:8 * c + 8].astype(np.float32)
                ws[g, :, 8 * c:8 * c + 8] = s[None, :] * (acc - z[None, :] * sumx[:, None])
    return ws.sum(0)


def dequant_like_the_kernel(qw, qz, sc, G, KK=64, CC=32, threads=256):
    K, Nq = qw.shape
    N = Nq * 8
    out = np.full((N, K), np.nan, np.float32)
    writes = np.zeros((N, K), np.int32)
    for by in range((K + KK - 1) // KK):
        for bx in range((Nq + CC - 1) // CC):
            k0, c0 = by * KK, bx * CC
            tile = np.zeros((KK, CC), np.int64)
            for t in range(threads):
                for r in range(KK * CC // threads):
                    kk, cc = t // CC + (threads // CC) * r, t % CC
                    k, c = k0 + kk, c0 + cc
                    tile[kk, cc] = qw[k, c] if (k < K and c < Nq) else 0
            for t in range(threads):
                kk = t % KK
                k = k0 + kk
                if k >= K:
                    continue
                g = k // G
                for r in range(CC // (threads // KK)):
                    cc = t // KK + (threads // KK) * r
                    c = c0 + cc
                    if c >= Nq:
                        break
                    q, z = unpack8(tile[kk, cc]), unpack8(qz[g, c])
                    for j in range(8):
                        out[8 * c + j, k] = (q[j] - z[j]) * np.float32(sc[g, 8 * c + j])
                        writes[8 * c + j, k] += 1
    return out, writes


def test_gemv_index_arithmetic():
    rng = torch.Generator().manual_seed(0)
    for N, K, G, M in ((72, 128, 32, 3), (520, 128, 64, 2)):      # 9 packed columns; a 1-thread last CTA
        w = torch.randn(N, K, generator=rng) * 0.05
        qw, qz, s = models.awq_quantize(w, G)
        x = torch.randn(M, K, generator=rng)
        got = gemv_like_the_kernel(x.numpy(), qw.numpy(), qz.numpy(), s.numpy(), G)
        want = (x @ loader.awq_dequant(qw, qz, s, G).t()).numpy()
        assert np.abs(got - want).max() < 1e-5 * max(1.0, np.abs(want).max())


def test_dequant_index_arithmetic():
    rng = torch.Generator().manual_seed(1)
    for N, K, G in ((72, 96, 32), (264, 64, 64)):                 # partial k tile; 33 packed columns
        w = torch.randn(N, K, generator=rng)
        qw, qz, s = models.awq_quantize(w, G)
        got, writes = dequant_like_the_kernel(qw.numpy(), qz.numpy(), s.numpy(), G)
        assert (writes == 1).all()
        assert np.array_equal(got, loader.awq_dequant(qw, qz, s, G).numpy())
