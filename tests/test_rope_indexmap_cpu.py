"""rope_qknorm_cache_kernel's index arithmetic (csrc/ops/elementwise.cu),
restated in numpy: a warp per head, lane l holding elements 2l, 2l+1 and
their rotation partners 2l+64, 2l+65; k and v written at the token's paged
slot. Against the fp32 reference rope(rmsnorm(head)). (The compiled kernel
is checked on the GPU in test_ops_gpu.py.)"""
import importlib

import numpy as np
import torch

ops = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops")
ref = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops.reference")


def kernel_like(qkv, pos, cs, slots, qn, kn, eps, nq, nkv, page, blocks, nwarps=8):
    T = qkv.shape[0]
    D, H2 = 128, 64
    q_out = np.zeros((T, nq, D), np.float32)
    kc = np.zeros((blocks, nkv, page, D), np.float32)
    vc = np.zeros_like(kc)
    for t in range(T):                                  # blockIdx.x
        c = cs[pos[t]]
        slot = slots[t]
        blk, off = slot // page, slot % page
        heads = nq + nkv if slot >= 0 else nq
        for warp in range(nwarps):
            for h in range(warp, heads, nwarps):
                src = qkv[t, h * D:(h + 1) * D]
                lanes = []
                for lane in range(32):
                    j = 2 * lane
                    a, b = src[j:j + 2], src[H2 + j:H2 + j + 2]
                    lanes.append((j, a, b))
                ss = sum(float((a * a).sum() + (b * b).sum()) for _, a, b in lanes)   # the warp reduction
                r = 1.0 / np.sqrt(ss / D + eps)
                w = qn if h < nq else kn
                for j, a, b in lanes:
                    a0, a1 = a[0] * r * w[j], a[1] * r * w[j + 1]
                    b0, b1 = b[0] * r * w[H2 + j], b[1] * r * w[H2 + j + 1]
                    c0, c1, s0, s1 = c[j], c[j + 1], c[H2 + j], c[H2 + j + 1]
                    y = [a0 * c0 - b0 * s0, a1 * c1 - b1 * s1, b0 * c0 + a0 * s0, b1 * c1 + a1 * s1]
                    dst = q_out[t, h] if h < nq else kc[blk, h - nq, off]
                    dst[j], dst[j + 1], dst[H2 + j], dst[H2 + j + 1] = y
        if slot >= 0:
            for kh in range(nkv):
                vc[blk, kh, off] = qkv[t, (nq + nkv + kh) * D:(nq + nkv + kh + 1) * D]
    return q_out, kc, vc


def test_rope_qknorm_index_arithmetic():
    g = torch.Generator().manual_seed(2)
    T, nq, nkv, D, page, blocks, eps = 5, 3, 2, 128, 16, 4, 1e-6
    qkv = torch.randn(T, (nq + 2 * nkv) * D, generator=g)
    pos = torch.tensor([0, 7, 3, 100, 41])
    cs = ops.rope_cos_sin(128, D, 1e6, "cpu")
    qn, kn = 1 + 0.3 * torch.randn(D, generator=g), 1 + 0.3 * torch.randn(D, generator=g)
    slots = torch.tensor([17, 3, 40, 63, 5])
    q, kc, vc = kernel_like(qkv.numpy(), pos.numpy(), cs.numpy(), slots.numpy(), qn.numpy(), kn.numpy(), eps,
                            nq, nkv, page, blocks)
    want_q = ref.rope(ref.rmsnorm(qkv[:, :nq * D].view(T, nq, D), qn, eps), pos, cs)
    want_k = ref.rope(ref.rmsnorm(qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D), kn, eps), pos, cs)
    assert np.abs(q - want_q.numpy()).max() < 1e-4
    blk, off = slots // page, slots % page
    assert np.abs(kc[blk.numpy(), :, off.numpy()] - want_k.numpy()).max() < 1e-4
    assert np.array_equal(vc[blk.numpy(), :, off.numpy()], qkv[:, (nq + nkv) * D:].view(T, nkv, D).numpy())
