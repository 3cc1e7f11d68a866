"""Plain PyTorch (fp32) references of every kernel, for numerics tests and the
cuBLAS/NCCL baseline model path. Shapes/semantics match ``ops``."""
import math

import torch
import torch.nn.functional as F


def gemm(a, w, residual=None):
    y = (a.float() @ w.float().t())
    if residual is not None:
        y = y.to(torch.bfloat16).float() + residual.float()
    return y


def rmsnorm(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def fused_add_rmsnorm(x, residual, w, eps):
    r = (x.float() + residual.float()).to(torch.bfloat16)
    return rmsnorm(r, w, eps), r


def rope(x, positions, cos_sin):
    """x [T, H, D]; neox rotation of the two halves."""
    D = x.shape[-1]
    cs = cos_sin[positions.long()]  # [T, D]
    c, s = cs[:, : D // 2].unsqueeze(1), cs[:, D // 2:].unsqueeze(1)
    x1, x2 = x.float()[..., : D // 2], x.float()[..., D // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def silu_mul(x):
    """silu(gate) rounded to bf16, times up (torch's bf16 evaluation order)."""
    g, u = x.float().chunk(2, dim=-1)
    return F.silu(g).to(torch.bfloat16).float() * u


def gather_kv(cache, block_table_row, length, page=16):
    """[length, nkv, D] from a paged cache [blocks, nkv, page, D]."""
    idx = torch.arange(length, device=cache.device)
    blk = block_table_row.long()[idx // page]
    return cache[blk, :, idx % page, :]


def attention(q, k, v, causal_offset=None):
    """q [Lq, nq, D], k/v [L, nkv, D]; query i at position causal_offset + i."""
    Lq, nq, D = q.shape
    L, nkv, _ = k.shape
    g = nq // nkv
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) / math.sqrt(D)
    if causal_offset is not None:
        qpos = torch.arange(Lq, device=q.device)[:, None] + causal_offset
        kpos = torch.arange(L, device=q.device)[None, :]
        s = s.masked_fill((kpos > qpos)[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vf)
