"""The served decoder's kernels restated in plain PyTorch, with the
signatures of ``ops``: fp32 math, bf16 results at the points where the CUDA
kernels round. Any device, CPU included.

It is the whole-engine oracle: ``LlamaTP(impl="oracle")`` and
``LLMEngine(impl="oracle")`` run the real scheduler, paged KV cache, prefix
cache, sampling and TP collectives (gloo on CPU) with these functions in
place of the CUDA kernels, so the engine's control paths are testable
without a GPU and the native engine can be compared with it token by token.
It is chosen only by that argument, never as a fallback for a missing
extension, and it is not a serving path.
"""
import torch

from . import reference as ref

BF16 = torch.bfloat16


def _emit(y, like_dtype, out):
    y = y.to(like_dtype)
    if out is None:
        return y
    out.copy_(y)
    return out


def gemm(a, w, out=None, residual=None, bn: int = 0, splits: int = 0):
    """out = a @ w^T (+ residual): fp32 accumulate, one bf16 rounding (two
    with a residual: the product, then the sum, as the fused epilogue)."""
    return _emit(ref.gemm(a, w, residual), BF16, out)


def awq_gemm(a, w, out=None, residual=None):
    """``ops.awq_gemm``: the int4 weight dequantized in fp32, then ``gemm``'s
    rounding."""
    from ..models.loader import awq_dequant

    dense = awq_dequant(w.qweight, w.qzeros, w.scales, w.group)
    return _emit(ref.gemm(a, dense, residual), BF16, out)


def rmsnorm(x, w, eps, out=None):
    return _emit(ref.rmsnorm(x, w, eps), x.dtype, out)


def fused_add_rmsnorm(x, residual, w, eps, out=None):
    """residual <- bf16(x + residual); returns rmsnorm(residual) * w."""
    y, r = ref.fused_add_rmsnorm(x, residual, w, eps)
    residual.copy_(r)
    return _emit(y, x.dtype, out)


def rope_and_cache(qkv, positions, cos_sin, nq, nkv, slots=None, k_cache=None, v_cache=None, q_out=None, page=16,
                   q_norm=None, k_norm=None, eps=0.0):
    """Rotate q/k of the fused [T, (nq + 2 nkv) D] projection (neox halves),
    store k/v at the paged ``slots`` (block * page + offset); returns q.
    ``q_norm`` / ``k_norm``: per-head RMSNorm of q and k first (Qwen3), kept
    in fp32 into the rotation."""
    T = qkv.shape[0]
    D = cos_sin.shape[1]
    q = qkv[:, :nq * D].view(T, nq, D)
    k = qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D)
    if q_norm is not None:
        q, k = ref.rmsnorm(q, q_norm, eps), ref.rmsnorm(k, k_norm, eps)
    v = qkv[:, (nq + nkv) * D:(nq + 2 * nkv) * D].view(T, nkv, D)
    qr = ref.rope(q, positions, cos_sin).to(qkv.dtype)
    if slots is not None:
        s = slots.long()
        blk, off = s // page, s % page
        k_cache[blk, :, off, :] = ref.rope(k, positions, cos_sin).to(k_cache.dtype)
        v_cache[blk, :, off, :] = v.to(v_cache.dtype)
    return _emit(qr, qkv.dtype, q_out)


def silu_mul(x, out=None):
    return _emit(ref.silu_mul(x), x.dtype, out)


def embedding(ids, table, start=0, out=None):
    """Rows of a vocab-parallel table; ids outside [start, start + rows) give 0."""
    local = ids.long() - start
    ok = (local >= 0) & (local < table.shape[0])
    y = torch.where(ok[:, None], table[local.clamp(0, table.shape[0] - 1)], torch.zeros((), dtype=table.dtype))
    return _emit(y, table.dtype, out)


def argmax(logits, offset=0, vals=None, idx=None):
    """Per row: (max value fp32, global index = offset + first maximal column)."""
    lf = logits.float()
    i = lf.argmax(-1)
    v = lf.gather(1, i[:, None])[:, 0]
    i = i + offset
    if vals is not None:
        vals.copy_(v)
        v = vals
    if idx is not None:
        idx.copy_(i)
        i = idx
    return v, i


def argmax_combine(vals, idx, out=None):
    """[ranks, B] per-shard maxima -> the global argmax per column (the
    lowest rank wins ties, i.e. the lowest vocabulary index)."""
    best = vals.argmax(0)
    return _emit(idx.gather(0, best[None])[0], torch.int64, out)


def paged_attention(q, k_cache, v_cache, q_lens, kv_lens, block_rows, page=16):
    """Causal attention of a ragged batch over the paged cache: request r's
    q_lens[r] queries are the last tokens of its kv_lens[r] cached keys.
    ``block_rows`` [R, max_blocks] int32. Scores are scaled by D^-1/2.
    Returns [T, nq, D] in q's dtype."""
    out = torch.empty_like(q)
    row = 0
    for r, (ql, kl) in enumerate(zip(q_lens, kv_lens)):
        k = ref.gather_kv(k_cache, block_rows[r], kl, page)
        v = ref.gather_kv(v_cache, block_rows[r], kl, page)
        out[row:row + ql] = ref.attention(q[row:row + ql], k, v, causal_offset=kl - ql).to(q.dtype)
        row += ql
    return out
