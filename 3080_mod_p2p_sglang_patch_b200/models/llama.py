"""Tensor-parallel Llama-style decoder on the package's sm_100a kernels.

Per rank (TP degree t): vocab-parallel embedding [V/t, H]; per layer a
column-parallel QKV [(nq+2nkv)/t*D, H] and gate_up [2F/t, H], row-parallel
o_proj [H, nq/t*D] and down [H, F/t]; vocab-parallel LM head [V/t, H].
Row-parallel outputs go through the communicator's fused
allreduce + residual add + RMSNorm (one launch), the point where the
reference's MailboxAR sits in sglang (RowParallelLinear ->
tensor_model_parallel_all_reduce, the call stack of its hot path).

``impl="native"``: tcgen05 GEMMs, own attention / norm / RoPE / SiLU kernels,
MailboxAR collectives. ``impl="torch"``: the NCCL(+cuBLAS) TP baseline -
F.linear (cuBLAS) GEMMs and NCCL allreduce, same attention/elementwise
kernels, so the two builds differ exactly in GEMMs and collectives.
``impl="oracle"``: every kernel restated in fp32 PyTorch (``ops.oracle``)
and plain torch.distributed collectives, on any device (CPU with gloo): the
whole-model oracle of the tests, not a serving path.
"""
import math

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..ops import oracle
from ..utils import nvtx
from .config import LlamaConfig


def _randn(shape, std, gen, device):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


class LlamaWeights:
    """Random-init N(0, std) weights of one TP rank.

    ``full_init=True`` draws every full tensor from one seeded generator and
    keeps this rank's shard (identical model at every TP degree, used by the
    tests); otherwise each shard is drawn directly from a seed derived from
    (seed, tensor, rank) (fast for 8B/70B)."""

    def __init__(self, cfg: LlamaConfig, tp_rank: int, tp_size: int, device, seed: int = 0, full_init: bool = False):
        cfg.check_tp(tp_size)
        self.cfg = cfg
        t, r = tp_size, tp_rank
        H, D, F_ = cfg.hidden, cfg.head_dim, cfg.ffn
        nq, nkv = cfg.heads // t, cfg.kv_heads // t
        V = cfg.vocab // t
        std = cfg.init_std
        dev = torch.device(device)
        counter = [0]

        def gen_for():
            counter[0] += 1
            g = torch.Generator(device=dev)
            g.manual_seed(seed * 1_000_003 + counter[0] * 7919 + (0 if full_init else r * 104_729))
            return g

        def col_parallel(full_rows_list, cols):
            # rows of several full matrices, this rank's slice of each, concatenated
            outs = []
            for full_rows in full_rows_list:
                g = gen_for()
                per = full_rows // t
                if full_init:
                    full = _randn((full_rows, cols), std, g, dev)
                    outs.append(full[r * per:(r + 1) * per])
                else:
                    outs.append(_randn((per, cols), std, g, dev))
            return torch.cat(outs, 0).contiguous()

        def row_parallel(rows, full_cols):
            g = gen_for()
            per = full_cols // t
            if full_init:
                full = _randn((rows, full_cols), std, g, dev)
                return full[:, r * per:(r + 1) * per].contiguous()
            return _randn((rows, per), std, g, dev)

        self.embed = col_parallel([cfg.vocab], H)
        self.layers = []
        for _ in range(cfg.layers):
            L = {}
            L["ln1"] = torch.ones(H, dtype=torch.bfloat16, device=dev)
            L["qkv"] = col_parallel([cfg.heads * D, cfg.kv_heads * D, cfg.kv_heads * D], H)
            L["o"] = row_parallel(H, cfg.heads * D)
            L["ln2"] = torch.ones(H, dtype=torch.bfloat16, device=dev)
            L["gate_up"] = col_parallel([F_, F_], H)
            L["down"] = row_parallel(H, F_)
            if cfg.qk_norm:  # Qwen3 per-head q/k norms, identity at init
                L["q_norm"] = torch.ones(D, dtype=torch.bfloat16, device=dev)
                L["k_norm"] = torch.ones(D, dtype=torch.bfloat16, device=dev)
            if cfg.qkv_bias:  # Qwen2 q/k/v biases, this rank's rows
                L["qkv_bias"] = col_parallel([cfg.heads * D, cfg.kv_heads * D, cfg.kv_heads * D], 1).view(-1)
            self.layers.append(L)
        self.norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.lm_head = col_parallel([cfg.vocab], H)
        self.vocab_start = r * V
        self.nq, self.nkv = nq, nkv


def _shard_weights(cfg: LlamaConfig, tp_rank: int, tp_size: int, device, fetch, linear=None):
    """A LlamaWeights whose shards come from ``fetch(name, rows=None, cols=None)``
    (full-tensor names as in Hugging Face Llama checkpoints, [out, in] layout;
    ``rows`` / ``cols`` = (start, stop) slices), converted to bf16 on ``device``.
    ``linear`` (same signature): a decoder linear's shard as an
    ``ops.Int4Weight``, or None to read it through ``fetch`` (int4 checkpoints
    kept packed)."""
    cfg.check_tp(tp_size)
    t, r = tp_size, tp_rank
    H, D, F_ = cfg.hidden, cfg.head_dim, cfg.ffn
    dev = torch.device(device)

    def get(name, rows=None, cols=None):
        return fetch(name, rows, cols).to(device=dev, dtype=torch.bfloat16).contiguous()

    def rows_of(name, full_rows):
        per = full_rows // t
        return get(name, rows=(r * per, (r + 1) * per))

    def cols_of(name, full_cols):
        per = full_cols // t
        return get(name, cols=(r * per, (r + 1) * per))

    def packed(names_rows):
        """Int4 shards of several column-parallel parts, concatenated; None
        unless every part is stored quantized."""
        if linear is None:
            return None
        parts = [linear(n, rows=(r * (f // t), (r + 1) * (f // t))) for n, f in names_rows]
        return ops.Int4Weight.cat(parts) if all(p is not None for p in parts) else None

    def packed_cols(name, full_cols):
        if linear is None:
            return None
        per = full_cols // t
        return linear(name, cols=(r * per, (r + 1) * per))

    w = LlamaWeights.__new__(LlamaWeights)
    w.cfg = cfg
    w.embed = rows_of("model.embed_tokens.weight", cfg.vocab)
    w.layers = []
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        L = {"ln1": get(p + "input_layernorm.weight"), "ln2": get(p + "post_attention_layernorm.weight")}
        if cfg.qk_norm:  # per-head norms: [head_dim], the same on every rank
            L["q_norm"] = get(p + "self_attn.q_norm.weight")
            L["k_norm"] = get(p + "self_attn.k_norm.weight")
        qkv_parts = [(p + "self_attn.q_proj.weight", cfg.heads * D), (p + "self_attn.k_proj.weight", cfg.kv_heads * D),
                     (p + "self_attn.v_proj.weight", cfg.kv_heads * D)]
        L["qkv"] = packed(qkv_parts)
        if L["qkv"] is None:
            L["qkv"] = torch.cat([rows_of(n, f) for n, f in qkv_parts], 0).contiguous()
        if cfg.qkv_bias:  # Qwen2: sharded like the projections' rows
            L["qkv_bias"] = torch.cat([rows_of(p + "self_attn.q_proj.bias", cfg.heads * D),
                                       rows_of(p + "self_attn.k_proj.bias", cfg.kv_heads * D),
                                       rows_of(p + "self_attn.v_proj.bias", cfg.kv_heads * D)], 0).contiguous()
        L["o"] = packed_cols(p + "self_attn.o_proj.weight", cfg.heads * D)
        if L["o"] is None:
            L["o"] = cols_of(p + "self_attn.o_proj.weight", cfg.heads * D)
        gu_parts = [(p + "mlp.gate_proj.weight", F_), (p + "mlp.up_proj.weight", F_)]
        L["gate_up"] = packed(gu_parts)
        if L["gate_up"] is None:
            L["gate_up"] = torch.cat([rows_of(n, f) for n, f in gu_parts], 0).contiguous()
        L["down"] = packed_cols(p + "mlp.down_proj.weight", F_)
        if L["down"] is None:
            L["down"] = cols_of(p + "mlp.down_proj.weight", F_)
        w.layers.append(L)
    w.norm = get("model.norm.weight")
    w.lm_head = rows_of("lm_head.weight", cfg.vocab)
    w.vocab_start = r * (cfg.vocab // t)
    w.nq, w.nkv = cfg.heads // t, cfg.kv_heads // t
    return w


class LlamaTP:
    """Forward passes of one TP rank over a paged KV cache.

    ``tp``: a ``parallel.TPGroup`` (or None for one GPU).
    """

    def __init__(self, cfg: LlamaConfig, weights: LlamaWeights, tp=None, impl: str = "native"):
        self.cfg = cfg
        self.w = weights
        self.tp = tp
        self.tp_size = tp.world_size if tp is not None else 1
        if impl not in ("native", "torch", "oracle"):
            raise ValueError(f"impl {impl!r}: native | torch | oracle")
        self.impl = impl
        # the elementwise / attention-side kernels: the CUDA ones, or their
        # fp32 restatements for the oracle
        self.k = oracle if impl == "oracle" else ops
        self.device = weights.embed.device
        self.cos_sin = ops.rope_cos_sin(cfg.max_pos, cfg.head_dim, cfg.rope_theta, self.device,
                                        dict(cfg.rope_scaling) if cfg.rope_scaling else None)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        # AWQ int4 layers (ops.Int4Weight): their GEMMs are not fused with the
        # collectives that follow them
        self.int4 = any(isinstance(v, ops.Int4Weight) for L in weights.layers for v in L.values())
        # sequence parallel (parallel/sp.py): used for batches of at least
        # ``sp_min_rows`` tokens that fit its buffers; None = off
        self.sp = None
        self.sp_min_rows = 256
        # overlapped micro-batches (``enable_overlap``): None = off
        self.overlap_min_rows = None
        self.overlap_threads = 256
        self._comm_stream = None

    def enable_sp(self, sp, min_rows: int = 256):
        """Run large batches sequence-parallel (native TP build, bf16 weights)."""
        if self.impl != "native" or self.tp_size == 1 or self.int4:
            return
        self.sp = sp
        self.sp_min_rows = int(min_rows)

    def enable_overlap(self, min_rows: int = 512, threads: int = 256):
        """Run native TP batches of at least ``min_rows`` tokens as two
        micro-batches on two streams, each with its own communication lane,
        so one micro-batch's allreduces run while the other computes (the
        caller passes per-micro-batch attention, see ``forward``).

        The reference's answer to the same problem is its segmented
        allreduce: the row-split GEMM output pushed by the copy engine while
        the next segment computes (sglang/mailbox_ar_ext.cu:233-342,
        docs/performance.md:51-65). Here whole layers overlap instead.
        ``threads=256`` launches the collectives with half-size blocks, which
        fit on an SM beside a GEMM CTA of the other micro-batch."""
        ca = self.tp.ca_comm if self.tp is not None else None
        ok = (self.impl == "native" and self.tp_size > 1 and not self.int4 and ca is not None
              and ca.lane() is not None)
        self.overlap_min_rows = int(min_rows) if ok else None
        self.overlap_threads = int(threads)

    def overlap_split(self, T: int):
        """Rows of the first micro-batch when a T-token batch runs overlapped
        (a multiple of 128 near T/2, the tile height of the GEMMs and the
        attention), else None."""
        if self.overlap_min_rows is None or T < self.overlap_min_rows:
            return None
        if self.sp is not None and T >= self.sp_min_rows and self.sp.fits(T):
            return None
        T1 = max(128, (T // 2) // 128 * 128)
        if T1 >= T:
            return None
        ca = self.tp.ca_comm
        nbytes = max(T1, T - T1) * self.cfg.hidden * 2
        if nbytes > ca.fused_rmsnorm_limit() or not ca.lane().fits_rmsnorm(nbytes):
            return None
        return T1

    def comm_stream(self):
        """The second micro-batch's stream (created once, high priority so its
        collectives get SMs as soon as they are free)."""
        if self._comm_stream is None:
            self._comm_stream = torch.cuda.Stream(device=self.device, priority=-1)
        return self._comm_stream

    # ------------------------------------------------------------ building blocks
    def _linear(self, x, w, out=None, residual=None):
        if isinstance(w, ops.Int4Weight):  # AWQ int4 kept packed
            if self.impl == "oracle":
                return oracle.awq_gemm(x, w, out=out, residual=residual)
            if self.impl != "native":
                raise ValueError("int4 weights run on the native build only")
            return ops.awq_gemm(x, w, out=out, residual=residual)
        if self.impl == "oracle":
            return oracle.gemm(x, w, out=out, residual=residual)
        if self.impl == "torch":
            y = F.linear(x, w)
            if residual is not None:
                y = y + residual
            if out is not None:
                out.copy_(y)
                return out
            return y
        return ops.gemm(x, w, out=out, residual=residual)

    def _all_reduce(self, x):
        if self.tp_size == 1:
            return x
        if self.impl == "oracle":  # fp32 sum, one rounding (gloo has no bf16 sum on every build)
            y = x.float()
            dist.all_reduce(y, group=self.tp.group)
            return x.copy_(y)
        if self.impl == "torch":
            dist.all_reduce(x, group=self.tp.group)
            return x
        return self.tp.all_reduce(x)

    def _ar_norm(self, partial, residual, w, out=None):
        """residual <- residual + allreduce(partial); returns rmsnorm(residual)."""
        if self.tp_size == 1 or self.impl != "native":
            x = self._all_reduce(partial)
            return self.k.fused_add_rmsnorm(x, residual, w, self.cfg.eps, out=out)
        return self.tp.all_reduce_rmsnorm(partial, residual, w, self.cfg.eps, out=out)

    def _qk_norm_args(self, L):
        """Qwen3's per-head q/k RMSNorm, applied by the RoPE kernel in the same
        launch (empty for Llama)."""
        if not self.cfg.qk_norm:
            return {}
        return {"q_norm": L["q_norm"], "k_norm": L["k_norm"], "eps": self.cfg.eps}

    def full_logits(self, x_last):
        """fp32 logits [B, V] over the whole vocabulary, identical on every
        rank (the LM-head shards all-gathered in rank order)."""
        logits = self._linear(x_last, self.w.lm_head)
        if self.tp_size == 1:
            return logits.float()
        B = logits.shape[0]
        if self.impl == "oracle":
            parts = [torch.empty_like(logits) for _ in range(self.tp_size)]
            dist.all_gather(parts, logits.contiguous(), group=self.tp.group)
            g = torch.stack(parts)
        elif self.impl == "torch":
            g = torch.empty((self.tp_size,) + tuple(logits.shape), dtype=logits.dtype, device=logits.device)
            dist.all_gather_into_tensor(g, logits.contiguous(), group=self.tp.group)
        else:
            g = self.tp.all_gather(logits.contiguous())  # [tp, B, V/tp]
        return g.permute(1, 0, 2).reshape(B, -1).float()

    def _lm_argmax(self, x_last):
        """Greedy next token from the vocab-parallel LM head."""
        logits = self._linear(x_last, self.w.lm_head)
        vals, idx = self.k.argmax(logits, offset=self.w.vocab_start)
        if self.tp_size == 1:
            return idx
        if self.impl == "oracle":
            gv = [torch.empty_like(vals) for _ in range(self.tp_size)]
            gi = [torch.empty_like(idx) for _ in range(self.tp_size)]
            dist.all_gather(gv, vals, group=self.tp.group)
            dist.all_gather(gi, idx, group=self.tp.group)
            return oracle.argmax_combine(torch.stack(gv), torch.stack(gi))
        if self.impl == "torch":
            gv = torch.empty((self.tp_size,) + vals.shape, dtype=vals.dtype, device=vals.device)
            gi = torch.empty((self.tp_size,) + idx.shape, dtype=idx.dtype, device=idx.device)
            dist.all_gather_into_tensor(gv, vals, group=self.tp.group)
            dist.all_gather_into_tensor(gi, idx, group=self.tp.group)
        else:
            # pack (val, idx) as two int64 words per row so one all-gather carries both
            B = vals.shape[0]
            pack = torch.empty((B, 2), dtype=torch.int64, device=vals.device)
            pack[:, 0] = vals.view(torch.int32).to(torch.int64)
            pack[:, 1] = idx
            g = self.tp.all_gather(pack)  # [tp, B, 2]
            gv = g[:, :, 0].to(torch.int32).view(torch.float32)
            gi = g[:, :, 1]
        return ops.argmax_combine(gv.contiguous(), gi.contiguous())

    # ------------------------------------------------------------ forward
    def forward(self, ids, positions, slots, kv_caches, attn, last_idx, return_hidden=False, attn_halves=None):
        """One forward over T tokens.

        ids/positions int32 [T]; slots int64 [T] (KV write slots); kv_caches
        [(k, v)] per layer; ``attn`` callable(layer, q, k_cache, v_cache) -> o
        [T, nq, D] (prefill or decode attention); last_idx int64 [B] rows whose
        next token is returned. Returns next-token ids int64 [B] (or the final
        normalised hidden rows [B, H] with ``return_hidden``).

        ``attn_halves``: (T1, attn0, attn1), attention of rows [0, T1) and
        [T1, T) on their own (attn1's keys include rows [0, T1), which the
        first micro-batch writes to the cache earlier in the same layer).
        Used when ``overlap_split(T) == T1``: the overlapped micro-batches.
        """
        cfg, w = self.cfg, self.w
        T = ids.shape[0]
        if self.sp is not None and T >= self.sp_min_rows and self.sp.fits(T):
            return self._forward_sp(ids, positions, slots, kv_caches, attn, last_idx, return_hidden)
        if attn_halves is not None and self.overlap_split(T) == attn_halves[0]:
            return self._forward_overlap(ids, positions, slots, kv_caches, attn_halves, last_idx, return_hidden)
        nq, nkv, D = w.nq, w.nkv, cfg.head_dim
        h = self.k.embedding(ids, w.embed, start=w.vocab_start)
        h = self._all_reduce(h)
        residual = h
        x = self.k.rmsnorm(residual, w.layers[0]["ln1"], cfg.eps)
        for li, L in enumerate(w.layers):
            if nvtx.ENABLED:
                torch.cuda.nvtx.range_push(f"layer {li}")
            kc, vc = kv_caches[li]
            q = None
            if self.impl == "native" and not cfg.qkv_bias and not self._qk_norm_args(L) and \
                    not isinstance(L["qkv"], ops.Int4Weight):
                # decode (1-2 tokens): projection, RoPE and cache writes in one GEMV launch
                q = ops.qkv_rope_and_cache(x, L["qkv"], positions, self.cos_sin, nq, nkv, slots, kc, vc)
            if q is None:
                qkv = self._linear(x, L["qkv"])
                if cfg.qkv_bias:
                    qkv += L["qkv_bias"]
                q = self.k.rope_and_cache(qkv, positions, self.cos_sin, nq, nkv, slots, kc, vc,
                                          **self._qk_norm_args(L))
            o = attn(li, q, kc, vc)
            if self.tp_size == 1 and self.impl == "native":
                # residual add fused into the GEMM epilogue, in place
                self._linear(o.view(T, nq * D), L["o"], out=residual, residual=residual)
                x = ops.rmsnorm(residual, L["ln2"], cfg.eps)
            elif self.impl == "native" and not isinstance(L["o"], ops.Int4Weight):
                # fused row-parallel GEMM -> allreduce -> residual + RMSNorm
                x = self.tp.gemm_all_reduce_rmsnorm(o.view(T, nq * D), L["o"], residual, L["ln2"], cfg.eps)
            else:
                part = self._linear(o.view(T, nq * D), L["o"])
                x = self._ar_norm(part, residual, L["ln2"])
            if self.impl == "native" and not isinstance(L["gate_up"], ops.Int4Weight):
                a = ops.gemm_silu(x, L["gate_up"])  # one GEMV launch at 1-2 rows
            else:
                a = self.k.silu_mul(self._linear(x, L["gate_up"]))
            nxt = w.layers[li + 1]["ln1"] if li + 1 < len(w.layers) else w.norm
            if self.tp_size == 1 and self.impl == "native":
                self._linear(a, L["down"], out=residual, residual=residual)
                x = ops.rmsnorm(residual, nxt, cfg.eps)
            elif self.impl == "native" and not isinstance(L["down"], ops.Int4Weight):
                x = self.tp.gemm_all_reduce_rmsnorm(a, L["down"], residual, nxt, cfg.eps)
            else:
                part = self._linear(a, L["down"])
                x = self._ar_norm(part, residual, nxt)
            if nvtx.ENABLED:
                torch.cuda.nvtx.range_pop()
        x_last = x.index_select(0, last_idx)
        if return_hidden:
            return x_last
        return self._lm_argmax(x_last)

    def _forward_overlap(self, ids, positions, slots, kv_caches, halves, last_idx, return_hidden=False):
        """Two micro-batches, rows [0, T1) and [T1, T), on two streams.

        Micro-batch 0 runs on the current stream with the communicator's main
        context, micro-batch 1 on a second stream with its second lane
        (``MailboxAR.lane``): each lane's collectives come in the same order on
        every rank, and the two lanes never share signal words, buffers or
        epochs. While one micro-batch waits in its allreduce + residual +
        RMSNorm, the other's GEMMs and attention use the SMs. The only
        cross-stream dependency per layer: micro-batch 1's attention reads the
        keys and values micro-batch 0 wrote to the cache for the same layer.
        Lane 1's kernels use their own scratch (``ops.workspace_lane``). Same
        math as ``forward`` row by row (sums in rank order, one rounding)."""
        cfg, w = self.cfg, self.w
        ca = self.tp.ca_comm
        lane1 = ca.lane()
        T1, attn0, attn1 = halves
        T = ids.shape[0]
        nq, nkv, D = w.nq, w.nkv, cfg.head_dim
        s0 = torch.cuda.current_stream(self.device)
        s1 = self.comm_stream()
        h = ops.embedding(ids, w.embed, start=w.vocab_start)
        residual = self._all_reduce(h)
        x = ops.rmsnorm(residual, w.layers[0]["ln1"], cfg.eps)
        part = torch.empty_like(residual)
        spans = ((0, T1), (T1, T))
        R = [residual[a:b] for a, b in spans]
        X = [x[a:b] for a, b in spans]
        P = [part[a:b] for a, b in spans]
        pos = [positions[a:b] for a, b in spans]
        sl = [slots[a:b] for a, b in spans]
        th = self.overlap_threads
        mb = ca.cfg.lane_max_blocks
        kv_ready = torch.cuda.Event()
        fork, join = torch.cuda.Event(), torch.cuda.Event()
        fork.record(s0)
        s1.wait_event(fork)

        def attn_block(i, li, L, kc, vc, attn):
            qkv = ops.gemm(X[i], L["qkv"])
            if cfg.qkv_bias:
                qkv += L["qkv_bias"]
            q = ops.rope_and_cache(qkv, pos[i], self.cos_sin, nq, nkv, sl[i], kc, vc, **self._qk_norm_args(L))
            if i == 0:
                kv_ready.record(s0)
            else:
                s1.wait_event(kv_ready)
            o = attn(li, q, kc, vc)
            ops.gemm(o.view(-1, nq * D), L["o"], out=P[i])

        def mlp_block(i, L):
            gu = ops.gemm(X[i], L["gate_up"])
            a = ops.silu_mul(gu)
            ops.gemm(a, L["down"], out=P[i])

        def collective(i, norm_w):
            if i == 0:
                ca.all_reduce_rmsnorm(P[0], R[0], norm_w, cfg.eps, out=X[0], threads=th, max_blocks=mb)
            else:
                lane1.all_reduce_rmsnorm(P[1], R[1], norm_w, cfg.eps, out=X[1], threads=th)

        for li, L in enumerate(w.layers):
            if nvtx.ENABLED:
                torch.cuda.nvtx.range_push(f"layer {li}")
            kc, vc = kv_caches[li]
            nxt = w.layers[li + 1]["ln1"] if li + 1 < len(w.layers) else w.norm
            attn_block(0, li, L, kc, vc, attn0)
            collective(0, L["ln2"])
            with torch.cuda.stream(s1), ops.workspace_lane(1):
                attn_block(1, li, L, kc, vc, attn1)
                collective(1, L["ln2"])
            mlp_block(0, L)
            collective(0, nxt)
            with torch.cuda.stream(s1), ops.workspace_lane(1):
                mlp_block(1, L)
                collective(1, nxt)
            if nvtx.ENABLED:
                torch.cuda.nvtx.range_pop()
        join.record(s1)
        s0.wait_event(join)
        x_last = x.index_select(0, last_idx)
        if return_hidden:
            return x_last
        return self._lm_argmax(x_last)

    def _forward_sp(self, ids, positions, slots, kv_caches, attn, last_idx, return_hidden=False):
        """Sequence-parallel forward: the residual stream is sharded by rows
        (this rank owns ``sp.own_rows(T)``); row-parallel GEMMs reduce-scatter
        from their epilogue, the owners normalise their rows and all-gather
        them into the gather buffer the next column-parallel GEMM loads from.
        Same math as ``forward`` (sums in rank order, one bf16 rounding)."""
        cfg, w, sp = self.cfg, self.w, self.sp
        T = ids.shape[0]
        nq, nkv, D = w.nq, w.nkv, cfg.head_dim
        h = ops.embedding(ids, w.embed, start=w.vocab_start)
        sp.rs_push(h)
        res = torch.zeros((sp.rows_per_rank(T), cfg.hidden), dtype=torch.bfloat16, device=ids.device)
        sp.rs_norm_ag(T, res, w.layers[0]["ln1"], cfg.eps)
        for li, L in enumerate(w.layers):
            qkv = sp.gemm_ag(T, L["qkv"])
            if cfg.qkv_bias:
                qkv += L["qkv_bias"]
            kc, vc = kv_caches[li]
            q = ops.rope_and_cache(qkv, positions, self.cos_sin, nq, nkv, slots, kc, vc, **self._qk_norm_args(L))
            o = attn(li, q, kc, vc)
            sp.gemm_rs(o.view(T, nq * D), L["o"])
            sp.rs_norm_ag(T, res, L["ln2"], cfg.eps)
            gu = sp.gemm_ag(T, L["gate_up"])
            a = ops.silu_mul(gu)
            sp.gemm_rs(a, L["down"])
            nxt = w.layers[li + 1]["ln1"] if li + 1 < len(w.layers) else w.norm
            sp.rs_norm_ag(T, res, nxt, cfg.eps)
        x_last = sp.gathered(T).index_select(0, last_idx)
        if return_hidden:
            return x_last
        return self._lm_argmax(x_last)
