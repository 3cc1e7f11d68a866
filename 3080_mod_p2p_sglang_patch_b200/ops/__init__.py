"""sm_100a kernels of the served decoder, as torch-tensor functions.

Every function dispatches to the in-tree CUDA extension; there is no PyTorch
fallback (a missing extension raises). Scratch memory (GEMM split-K partials,
decode split-KV partials, the GEMM error word) comes from a per-device
workspace that is allocated once and reused, so CUDA-graph capture never
allocates.
"""
import contextlib
import dataclasses
import math

import os

import torch

from .._ext import cuda_ext
from ..utils import launches


class _Workspace:
    """Scratch buffers of one device. A buffer that must grow is replaced by
    a new, larger one and the old one is kept alive (``_retired``): a CUDA graph
    that captured the old address keeps valid memory."""

    def __init__(self, device, err=None):
        self.device = device
        self.err = err if err is not None else torch.zeros(1, dtype=torch.int32, device=device)
        # arrival counters of in-kernel merges (split-KV decode attention; each
        # reset by the last CTA that arrives)
        self.counters = torch.zeros(65536, dtype=torch.int32, device=device)
        self.gemm_ws = torch.empty(0, dtype=torch.float32, device=device)
        self.dec_o = torch.empty(0, dtype=torch.float32, device=device)
        self.dec_lse = torch.empty(0, dtype=torch.float32, device=device)
        self.pre_o = torch.empty(0, dtype=torch.float32, device=device)
        self.pre_lse = torch.empty(0, dtype=torch.float32, device=device)
        self.awq_ws = torch.empty(0, dtype=torch.float32, device=device)    # int4 GEMV partial sums
        self.awq_w = torch.empty(0, dtype=torch.bfloat16, device=device)    # one layer dequantized
        self._retired = []

    def _grow(self, name, n, minimum, dtype=torch.float32):
        buf = getattr(self, name)
        if buf.numel() < n:
            if buf.numel():
                self._retired.append(buf)
            buf = torch.empty(max(n, minimum), dtype=dtype, device=self.device)
            setattr(self, name, buf)
        return buf

    def gemm(self, n):
        return self._grow("gemm_ws", n, 1 << 22)

    def decode(self, n_o, n_lse):
        return self._grow("dec_o", n_o, 1 << 20), self._grow("dec_lse", n_lse, 1 << 14)

    def prefill(self, n_o, n_lse):
        return self._grow("pre_o", n_o, 1 << 20), self._grow("pre_lse", n_lse, 1 << 14)

    def awq(self, n_ws=0, n_w=0):
        return self._grow("awq_ws", n_ws, 1 << 16), self._grow("awq_w", n_w, 1 << 16, torch.bfloat16)


_WS = {}
_LANE = [0]


@contextlib.contextmanager
def workspace_lane(lane: int):
    """Kernels launched inside use lane ``lane``'s scratch buffers. Work issued
    on a second stream that runs at the same time as the first (the
    overlapped micro-batches) must not share the split-K or split-KV partial
    buffers; the error word is shared by all lanes."""
    prev = _LANE[0]
    _LANE[0] = int(lane)
    try:
        yield
    finally:
        _LANE[0] = prev


def workspace(device) -> _Workspace:
    key = torch.device(device).index
    if key is None:
        key = torch.cuda.current_device()
    lane = _LANE[0]
    ws = _WS.get((key, lane))
    if ws is None:
        dev = torch.device("cuda", key)
        base = _WS.get((key, 0)) if lane else None
        if lane and base is None:
            base = _WS[(key, 0)] = _Workspace(dev)
        ws = _WS[(key, lane)] = _Workspace(dev, err=base.err if base is not None else None)
    return ws


def reserve(device, gemm_elems=0, decode_o=0, decode_lse=0, awq_ws=0, awq_w=0):
    """Pre-size the scratch buffers (call before CUDA-graph capture)."""
    ws = workspace(device)
    if gemm_elems:
        ws.gemm(gemm_elems)
    if decode_o or decode_lse:
        ws.decode(decode_o, decode_lse)
    if awq_ws or awq_w:
        ws.awq(awq_ws, awq_w)


def gemm_error(device=None) -> int:
    """Non-zero if a tcgen05 kernel's bounded wait gave up (GEMM or prefill
    attention; sticky until cleared)."""
    return int(workspace(device or torch.cuda.current_device()).err.item())


def gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor = None, residual: torch.Tensor = None,
         bn: int = 0, splits: int = 0) -> torch.Tensor:
    """out[M, N] = a[M, K] @ w[N, K]^T (+ residual): the tcgen05/TMEM kernel,
    or for 1-2 rows (decode) the CUDA-core GEMV, a plain weight stream."""
    C = cuda_ext()
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    ws = workspace(a.device)
    plan_bn, plan_splits = C.gemm_plan(M, N, K)
    s = splits or plan_splits
    wbuf = ws.gemm(s * M * N) if s > 1 else None
    # split-K partials are folded by a separate reduce kernel: the in-kernel
    # reduction (pass ws.counters) measured no faster at 1 token, slower at 64,
    # and 1.5-2x slower at 512-1024 rows (qkv at TP=4/8)
    C.gemm(a, w, out, residual, wbuf, ws.err, bn, splits, None)
    gemv = M <= C.GEMV_MAX_ROWS and not bn and not splits and K % 8 == 0 and _GEMV_ON
    launches.add(1 if gemv or s <= 1 else 2)
    return out


_GEMV_ON = os.environ.get("MBX_GEMV", "1") != "0"
_DECODE_MERGE = os.environ.get("MBX_DECODE_MERGE", "1") != "0"


@dataclasses.dataclass
class Int4Weight:
    """A linear layer's weight kept as AWQ int4 (``gemm`` packing): qweight
    int32 [K, N/8], qzeros int32 [K/G, N/8], scales fp16 [K/G, N]. ``shape``
    is the dense weight's [N, K], as for a bf16 weight."""
    qweight: torch.Tensor
    qzeros: torch.Tensor
    scales: torch.Tensor
    group: int

    @property
    def shape(self):
        return (self.qweight.shape[1] * 8, self.qweight.shape[0])

    @property
    def device(self):
        return self.qweight.device

    @staticmethod
    def cat(parts):
        """Concatenated along the output dimension (fused qkv / gate_up)."""
        g = {p.group for p in parts}
        if len(g) != 1:
            raise ValueError("int4 weights with different group sizes")
        return Int4Weight(torch.cat([p.qweight for p in parts], 1).contiguous(),
                          torch.cat([p.qzeros for p in parts], 1).contiguous(),
                          torch.cat([p.scales for p in parts], 1).contiguous(), g.pop())


AWQ_GEMV_MAX_ROWS = 8     # rows per int4 GEMV launch
# up to this many rows the int4 GEMV runs (in 8-row chunks); above it the layer
# is dequantized for the tcgen05 GEMM. Measured on 8B decode at TP=1: 16 rows
# 11.7 ms per step dequantized vs 15.6 ms as two GEMV chunks; 64 rows 15.8 vs
# 58.3 (MBX_AWQ_GEMV_ROWS overrides)
AWQ_GEMV_ROW_LIMIT = int(os.environ.get("MBX_AWQ_GEMV_ROWS", "8"))


def awq_gemm(a: torch.Tensor, w: Int4Weight, out: torch.Tensor = None, residual: torch.Tensor = None):
    """out[M, N] = a @ W^T (+ residual) for an int4 weight.

    Up to AWQ_GEMV_ROW_LIMIT rows (small decode batches): the int4 GEMV, which
    reads the packed weight once (a quarter of bf16's bytes) and does its
    math on the CUDA cores. Larger batches: the layer dequantized to bf16
    into a reused scratch buffer and the tcgen05 GEMM (the expansion costs
    about 2.25x the bf16 weight bytes)."""
    C = cuda_ext()
    M = a.shape[0]
    N, K = w.shape
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    ws = workspace(a.device)
    if M <= AWQ_GEMV_ROW_LIMIT and w.group <= 256 and w.group % 32 == 0:
        part, _ = ws.awq(n_ws=(K // w.group) * min(M, AWQ_GEMV_MAX_ROWS) * N)
        for r0 in range(0, M, AWQ_GEMV_MAX_ROWS):
            r1 = min(M, r0 + AWQ_GEMV_MAX_ROWS)
            C.awq_gemv(a[r0:r1], w.qweight, w.qzeros, w.scales, w.group, part, out[r0:r1],
                       None if residual is None else residual[r0:r1])
            launches.add(2)
        return out
    _, wbuf = ws.awq(n_w=N * K)
    dense = wbuf[:N * K].view(N, K)
    C.awq_dequant(w.qweight, w.qzeros, w.scales, w.group, dense)
    launches.add(1)
    return gemm(a, dense, out=out, residual=residual)


def awq_dequant(w: Int4Weight) -> torch.Tensor:
    """bf16 [N, K] copy of an int4 weight (a new tensor)."""
    N, K = w.shape
    out = torch.empty((N, K), dtype=torch.bfloat16, device=w.device)
    cuda_ext().awq_dequant(w.qweight, w.qzeros, w.scales, w.group, out)
    launches.add(1)
    return out


def rmsnorm(x, w, eps, out=None):
    out = torch.empty_like(x) if out is None else out
    cuda_ext().rmsnorm(x, w, out, eps)
    launches.add(1)
    return out


def fused_add_rmsnorm(x, residual, w, eps, out=None):
    """residual <- bf16(x + residual); returns rmsnorm(residual) * w."""
    out = torch.empty_like(x) if out is None else out
    cuda_ext().fused_add_rmsnorm(x, residual, w, out, eps)
    launches.add(1)
    return out


# rope_scaling types rope_cos_sin implements (None / "default": plain RoPE)
ROPE_SCALINGS = (None, "default", "linear", "llama3")


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, device, scaling=None) -> torch.Tensor:
    """[max_pos, head_dim] fp32 table: cos in the first half, sin in the second.

    ``scaling`` (dict) with ``rope_type == "linear"`` divides every frequency
    by ``factor`` (position interpolation); other types raise.

    ``scaling`` (dict) with ``rope_type == "llama3"`` applies Llama 3.1's
    frequency rescaling: wavelengths above original_max_position /
    low_freq_factor are divided by ``factor``, those below original /
    high_freq_factor are kept, and the band between is interpolated linearly
    in original / wavelength."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    kind = scaling.get("rope_type", scaling.get("type")) if scaling else None
    if kind not in ROPE_SCALINGS:
        raise ValueError(f"rope scaling {kind!r} is not supported (supported: {', '.join(map(str, ROPE_SCALINGS))})")
    if kind == "linear":  # position interpolation: every frequency divided by the factor
        inv = inv / float(scaling["factor"])
    if kind == "llama3":
        factor = float(scaling["factor"])
        lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        orig = float(scaling.get("original_max_position_embeddings", 8192))
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        inv = torch.where(wavelen > orig / lo, inv / factor,
                          torch.where(wavelen < orig / hi, inv, (1 - smooth) * inv / factor + smooth * inv))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).to(torch.float32).to(device)


def rope_and_cache(qkv, positions, cos_sin, nq, nkv, slots=None, k_cache=None, v_cache=None, q_out=None, page=16,
                   q_norm=None, k_norm=None, eps=0.0):
    """Rotate q/k (neox), write rotated q to q_out [T, nq, 128] and k/v to the
    paged cache at ``slots`` (int64 block*page+offset). ``q_norm`` /
    ``k_norm`` (bf16 [128]): Qwen3's per-head RMSNorm of q and k (epsilon
    ``eps``) before the rotation, in the same launch."""
    T = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty((T, nq, 128), dtype=qkv.dtype, device=qkv.device)
    cuda_ext().rope_and_cache(qkv, positions, cos_sin, slots, q_out, k_cache, v_cache, nq, nkv, page, q_norm, k_norm,
                              float(eps))
    launches.add(1)
    return q_out


def silu_mul(x, out=None):
    if out is None:
        out = torch.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=x.dtype, device=x.device)
    cuda_ext().silu_mul(x, out)
    launches.add(1)
    return out


def qkv_rope_and_cache(x, w, positions, cos_sin, nq, nkv, slots=None, k_cache=None, v_cache=None, page=16):
    """The attention input of decode: q = RoPE(x @ Wq^T) and the paged k/v
    writes, in one GEMV launch for 1-2 tokens (no q/k norm, no bias); None
    when the shape does not fit it (the caller runs gemm + rope_and_cache,
    which round the same way)."""
    C = cuda_ext()
    T = x.shape[0]
    if T > C.GEMV_MAX_ROWS or not _GEMV_ON:
        return None
    q_out = torch.empty((T, nq, 128), dtype=torch.bfloat16, device=x.device)
    if not C.gemv_rope(x, w, positions, cos_sin, slots, q_out, k_cache, v_cache, nq, nkv, page):
        return None
    launches.add(1)
    return q_out


def gemm_silu(x, w, out=None):
    """silu(x @ gate^T) * (x @ up^T) for a gate_up weight [2F, K] (gate rows
    first): one GEMV launch for 1-2 rows (decode), else the GEMM and
    silu_mul. Same roundings either way."""
    M, F = x.shape[0], w.shape[0] // 2
    if out is None:
        out = torch.empty((M, F), dtype=torch.bfloat16, device=x.device)
    if M <= cuda_ext().GEMV_MAX_ROWS and _GEMV_ON and cuda_ext().gemv_silu(x, w, out):
        launches.add(1)
        return out
    return silu_mul(gemm(x, w), out=out)


def embedding(ids, table, start=0, out=None):
    if out is None:
        out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device)
    cuda_ext().embedding(ids, table, out, start)
    launches.add(1)
    return out


def argmax(logits, offset=0, vals=None, idx=None):
    B = logits.shape[0]
    if vals is None:
        vals = torch.empty(B, dtype=torch.float32, device=logits.device)
    if idx is None:
        idx = torch.empty(B, dtype=torch.int64, device=logits.device)
    cuda_ext().argmax(logits, offset, vals, idx)
    launches.add(1)
    return vals, idx


def argmax_combine(vals, idx, out=None):
    if out is None:
        out = torch.empty(vals.shape[1], dtype=torch.int64, device=vals.device)
    cuda_ext().argmax_combine(vals, idx, out)
    launches.add(1)
    return out


PREFILL_BQ = 256  # query rows per CTA of the tcgen05 prefill kernel (two 128-row tiles)


def prefill_tiles(q_lens, bq: int = PREFILL_BQ):
    """(request, q offset) pairs of the query tiles of a ragged batch, the
    tiles with the most keys first (causal: later tiles see more keys)."""
    tiles = []
    for r, n in enumerate(q_lens):
        for off in range(0, n, bq):
            tiles.append((r, off))
    tiles.sort(key=lambda t: -t[1])
    return torch.tensor(tiles, dtype=torch.int32).reshape(-1, 2)


def prefill_splits(n_tiles: int, nq: int, max_kv: int, sms: int = 148) -> int:
    """Split-KV factor for the prefill kernel. Splitting costs a partial
    write plus a combine pass, which only pays when fewer than half the SMs
    would be busy (high TP: few heads per rank); then enough splits to cover
    the SMs, at least 512 keys per split."""
    ctas = max(1, n_tiles * nq)
    if 2 * ctas > sms:
        return 1
    want = -(-sms // ctas)
    return int(max(1, min(want, max_kv // 512, 16)))


def prefill_attention(q, k_cache, v_cache, cu_q, kv_len, block_table, tiles, scale=None, out=None, splits=1):
    """Causal chunked-prefill attention over the paged cache, tcgen05/TMEM
    kernel; ``tiles`` from ``prefill_tiles(q_lens)`` (128-row tiles).
    ``splits`` > 1 splits each query tile's keys across CTAs (see
    ``prefill_splits``); the partials are merged by a combine kernel."""
    if out is None:
        out = torch.empty_like(q)
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    po = pl = None
    if splits > 1:
        T, nq, _ = q.shape
        po, pl = workspace(q.device).prefill(T * nq * splits * 128, T * nq * splits)
    cuda_ext().prefill_attention_tc(q, k_cache, v_cache, out, cu_q, kv_len, block_table, tiles, scale,
                                    workspace(q.device).err, splits, po, pl)
    launches.add(2 if splits > 1 else 1)
    return out


def prefill_attention_mma(q, k_cache, v_cache, cu_q, kv_len, block_table, tiles64, scale=None, out=None):
    """The same attention with legacy mma.sync (m16n8k16) tensor-core MMAs;
    ``tiles64`` from ``prefill_tiles(q_lens, bq=64)``. Kept as the baseline
    the tcgen05 kernel is measured against."""
    if out is None:
        out = torch.empty_like(q)
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    cuda_ext().prefill_attention(q, k_cache, v_cache, out, cu_q, kv_len, block_table, tiles64, scale)
    launches.add(1)
    return out


def decode_splits(batch: int, nkv: int, max_len: int, sms: int = 148) -> int:
    """Split-KV factor so (batch x kv-heads x splits) fills the SMs, with at
    least 16 pages (256 keys) per split: finer splits cost more in the LSE
    combine than they gain (measured at batch 1, context 4096)."""
    want = max(1, (2 * sms) // max(1, batch * nkv))
    by_len = max(1, max_len // 256)
    return int(min(want, by_len, 64))


def decode_attention(q, k_cache, v_cache, kv_len, block_table, scale=None, splits=1, out=None):
    if out is None:
        out = torch.empty_like(q)
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, nq, _ = q.shape
    po = pl = cnt = None
    if splits > 1:
        ws = workspace(q.device)
        po, pl = ws.decode(B * nq * splits * 128, B * nq * splits)
        # the last CTA of each (request, kv head) merges the splits in the kernel
        # (MBX_DECODE_MERGE=0: a separate combine launch)
        cnt = ws.counters if _DECODE_MERGE and B * k_cache.shape[1] <= ws.counters.numel() else None
    cuda_ext().decode_attention(q, k_cache, v_cache, out, kv_len, block_table, po, pl, splits, scale, cnt)
    launches.add(2 if splits > 1 and cnt is None else 1)
    return out
