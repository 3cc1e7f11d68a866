"""Offline serving engine: chunked prefill (optionally with decode tokens
mixed in) and CUDA-graph decode.

``LLMEngine(cfg, tp=TPGroup|None, ...)`` owns one TP rank's weights, paged KV
cache (optionally shared prefixes), scheduler and graph runners. Every TP
rank runs the same deterministic schedule, so all ranks take the same
collective steps.

Public API:

* ``generate(prompts, max_new_tokens, stop_ids, sampling)``: token ids in,
  token ids out. With ``max_new_tokens=1`` it is the prefill measurement of
  the reference's prompt-processing bench (tests/pp_bench.py).
* ``generate_text(prompts, sampling_params)``: text in the shape of sglang's
  offline engine.
* ``add_request`` / ``step`` / ``run`` / ``abort`` for streaming use. Requests
  can ask for sampling, logit adjustments, logprobs or prompt scoring.
* ``from_pretrained(dir, ...)`` for Hugging Face checkpoints.
"""
import os
import time

import torch

from .. import ops
from ..ops import oracle
from ..utils import nvtx
from ..models import LlamaConfig, LlamaTP, LlamaWeights
from .graph_runner import DecodeGraphRunner, PrefillGraphRunner
from .kv_cache import PAGE, PagedKVCache, PrefixCache
from .sampling import GREEDY, SamplingParams, adjust_logits, sample
from .scheduler import Request, Scheduler


class LLMEngine:
    def __init__(self, cfg: LlamaConfig, tp=None, max_batch: int = 64, max_seq: int = 8192, chunk: int = 1024,
                 seed: int = 0, use_graphs: bool = True, impl: str = "native", kv_blocks: int = None,
                 graph_sizes=(1, 8, 32, 64), full_init: bool = False, device=None, prefill_graph: bool = False,
                 sp: bool = None, weights=None, prefix_cache: bool = False, mem_fraction: float = None,
                 mixed_chunk: bool = False, schedule_policy: str = "fcfs", sample_in_graphs: bool = False,
                 overlap: bool = None, overlap_min_rows: int = 512):
        if impl == "oracle":  # fp32 torch restatement of every kernel: eager, any device
            use_graphs, prefill_graph = False, False
        if max_seq > cfg.max_pos:
            # positions index the RoPE table, which has max_pos rows
            raise ValueError(f"max_seq {max_seq} exceeds the model's {cfg.max_pos} positions")
        self.cfg = cfg
        self.tp = tp
        self.impl = impl
        # decode batches that need the full logits (sampling, logprobs, logit
        # adjustments) replay a CUDA graph ending in the logits instead of
        # running eagerly
        self.sample_in_graphs = sample_in_graphs
        # text API (generate_text): the checkpoint's tokenizer and stop ids when
        # loaded with from_pretrained, else bytes and none
        self.tokenizer = None
        self.default_stop_ids = ()
        self.tp_size = tp.world_size if tp is not None else 1
        self.tp_rank = tp.rank if tp is not None else 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_batch = max_batch
        self.max_seq = max_seq
        self.chunk = chunk
        # random-init weights unless a checkpoint's shards are given (models.load_llama)
        self.weights = weights if weights is not None else LlamaWeights(cfg, self.tp_rank, self.tp_size, self.device,
                                                                        seed=seed, full_init=full_init)
        self.model = LlamaTP(cfg, self.weights, tp=tp, impl=impl)
        # sequence parallel for prefill batches (TP > 1, native build);
        # None = follow MBX_SP (default off)
        if sp is None:
            sp = os.environ.get("MBX_SP", "0") == "1"
        self.sp = None
        if sp and tp is not None and self.tp_size > 1 and impl == "native":
            self.sp = tp.sp_setup(chunk, cfg.hidden)
            if self.sp is not None:
                self.model.enable_sp(self.sp)
        # overlapped micro-batches for large prefill batches (TP > 1, native
        # build): each micro-batch's allreduces run while the other computes;
        # None = follow MBX_OVERLAP (default off)
        if overlap is None:
            overlap = os.environ.get("MBX_OVERLAP", "0") == "1"
        self.overlap = False
        if overlap and tp is not None and self.tp_size > 1 and impl == "native":
            self.model.enable_overlap(min_rows=overlap_min_rows)
            self.overlap = self.model.overlap_min_rows is not None
        nkv = cfg.kv_heads // self.tp_size
        self.max_blocks_per_seq = (max_seq + PAGE - 1) // PAGE
        if kv_blocks is None:
            kv_blocks = max_batch * self.max_blocks_per_seq + 1
            if mem_fraction is not None and self.device.type == "cuda":
                # weights + KV cache within mem_fraction of the device (the rest:
                # activations, workspaces, CUDA graphs)
                free, total = torch.cuda.mem_get_info(self.device)
                block_bytes = PagedKVCache.bytes_per_token(cfg.layers, nkv, cfg.head_dim) * PAGE
                fit = PagedKVCache.blocks_for_memory(total, free, mem_fraction, block_bytes)
                if fit < self.max_blocks_per_seq:
                    raise ValueError(f"mem_fraction {mem_fraction}: the KV cache would hold {fit * PAGE} tokens, "
                                     f"fewer than max_seq {max_seq}")
                kv_blocks = min(kv_blocks, fit + 1)
        self.kv = PagedKVCache(cfg.layers, nkv, cfg.head_dim, kv_blocks, self.device)
        # prefix caching: off by default (benchmarks must not reuse work)
        self.prefix_cache = PrefixCache(self.kv.alloc) if prefix_cache else None
        self.sched = Scheduler(chunk, max_batch, self.kv.alloc, max_seq, prefix_cache=self.prefix_cache,
                               mixed=mixed_chunk, policy=schedule_policy)
        # draws of unseeded sampled requests (same seed on every TP rank)
        self._rng = torch.Generator(device=self.device)
        self._rng.manual_seed(int(seed) + 1_000_003)
        self.block_table = torch.zeros((max_batch, self.max_blocks_per_seq), dtype=torch.int32, device=self.device)
        self._next_rid = 0
        # scratch sized once (graph capture must not allocate)
        self._reserve_scratch()
        self.graphs = None
        self.prefill_graph = None
        if use_graphs:
            sizes = tuple(s for s in graph_sizes if s <= max_batch)
            self.graphs = DecodeGraphRunner(self, sizes)
        if prefill_graph:
            self.prefill_graph = PrefillGraphRunner(self, chunk)

    def _sample_tokens(self, hidden, reqs, draw=None):
        """Next tokens for rows of final hidden states (one per request).
        ``draw[i]`` False: row i's token is not used (a prefill piece that
        does not end its prompt), so it is taken greedily and no generator
        advances."""
        return self._sample_from_logits(self.model.full_logits(hidden), reqs, draw)

    def _sample_from_logits(self, logits, reqs, draw=None):
        raw = logits
        if any(r.sampling is not None and r.sampling.adjusts for r in reqs):
            logits = adjust_logits(logits, [r.sampling for r in reqs], [r.prompt for r in reqs],
                                   [r.output for r in reqs], [r.stop_ids for r in reqs])
        params, gens = [], []
        for i, r in enumerate(reqs):
            use = r.sampled and (draw is None or draw[i])
            params.append(r.sampling if use else GREEDY)  # adjustments are already in the logits
            gens.append((r.rng if r.rng is not None else self._rng) if use else None)
        tokens = sample(logits, params, gens)
        want = [i for i, r in enumerate(reqs) if r.logprobs is not None and (draw is None or draw[i])]
        if want:
            # logprobs of the model's own distribution (before penalties, temperature, top-k / top-p)
            rows = torch.tensor(want, device=raw.device)
            lp = torch.log_softmax(raw.index_select(0, rows).float(), dim=-1)
            chosen = lp.gather(1, tokens.index_select(0, rows)[:, None])[:, 0].tolist()
            k = max(reqs[i].logprobs for i in want)
            top_v, top_i = torch.topk(lp, k, dim=-1) if k > 0 else (lp[:, :0], lp[:, :0].long())
            top_v, top_i = top_v.tolist(), top_i.tolist()
            for j, i in enumerate(want):
                n = reqs[i].logprobs
                reqs[i].token_logprobs.append((chosen[j], list(zip(top_i[j][:n], top_v[j][:n]))))
        return tokens

    @classmethod
    def from_pretrained(cls, model_dir: str, tp=None, device=None, **kw):
        """Engine over a Hugging Face checkpoint directory (this rank's shards
        only are read; see models/loader.py). ``int4_weights=True`` keeps an
        AWQ checkpoint's linears packed (int4 GEMV for decode batches, a
        per-layer bf16 expansion for prefill) instead of expanding them once.
        ``tokenizer_path``: load the tokenizer from another directory."""
        from ..models.loader import load_llama, stop_token_ids
        from .tokenizer import HFTokenizer

        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        int4 = bool(kw.pop("int4_weights", False))
        tok_dir = kw.pop("tokenizer_path", None) or model_dir
        cfg, w = load_llama(model_dir, tp.rank if tp is not None else 0, tp.world_size if tp is not None else 1, dev,
                            int4=int4)
        kw.setdefault("max_seq", min(cfg.max_pos, 8192))
        eng = cls(cfg, tp=tp, device=dev, weights=w, **kw)
        try:
            eng.tokenizer = HFTokenizer(tok_dir)
        except Exception:  # noqa: BLE001 - token-id APIs still work without one
            if tok_dir != model_dir:  # asked for explicitly: not silently dropped
                raise
            eng.tokenizer = None
        eng.default_stop_ids = stop_token_ids(model_dir)
        return eng

    @property
    def max_request_tokens(self) -> int:
        """Longest prompt + max_new_tokens one request may have: max_seq, or
        less if the KV cache is smaller than that."""
        return min(self.max_seq, self.kv.alloc.capacity * PAGE)

    # ------------------------------------------------------------------ setup
    def _h2d(self, host: torch.Tensor) -> torch.Tensor:
        """A host tensor on the engine's device (pinned, asynchronous on CUDA)."""
        if self.device.type != "cuda":
            return host.to(self.device)
        return host.pin_memory().to(self.device, non_blocking=True)

    def _reserve_scratch(self):
        if self.impl == "oracle" or self.device.type != "cuda":
            return
        cfg, t = self.cfg, self.tp_size
        C = None
        try:
            from .._ext import cuda_ext

            C = cuda_ext()
        except Exception:  # noqa: BLE001
            return
        H, F_, D = cfg.hidden, cfg.ffn // t, cfg.head_dim
        shapes = [((cfg.heads + 2 * cfg.kv_heads) // t * D, H), (H, cfg.heads // t * D), (2 * F_, H), (H, F_),
                  (cfg.vocab // t, H)]
        need = 0
        for M in (1, 8, 32, 64, self.max_batch, self.chunk):
            for N, K in shapes:
                bn, splits = C.gemm_plan(M, N, K)
                if splits > 1:
                    need = max(need, splits * M * N)
        nq = cfg.heads // t
        max_splits = 64
        awq_ws = awq_w = 0
        for L in self.weights.layers[:1]:  # every layer has the same shapes
            for w in L.values():
                if isinstance(w, ops.Int4Weight):
                    N_, K_ = w.shape
                    awq_ws = max(awq_ws, (K_ // w.group) * ops.AWQ_GEMV_MAX_ROWS * N_)
                    awq_w = max(awq_w, N_ * K_)
        ops.reserve(self.device, gemm_elems=need, decode_o=self.max_batch * nq * max_splits * D,
                    decode_lse=self.max_batch * nq * max_splits, awq_ws=awq_ws, awq_w=awq_w)

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt, max_new_tokens: int, stop_ids=(), sampling=None, logprobs: int = None,
                    prompt_logprobs: bool = False) -> Request:
        """Queue a prompt (token ids); generation ends after ``max_new_tokens``
        or after any token in ``stop_ids`` (kept in the output). ``sampling``:
        a SamplingParams (None = greedy); a seeded one draws from its own
        generator, an unseeded one from the engine's (seeded identically on
        every TP rank, so all ranks draw the same tokens). ``logprobs`` k:
        record each generated token's logprob and the k most likely
        alternatives in ``request.token_logprobs`` (such requests run eagerly,
        with full logits). ``prompt_logprobs``: also score the prompt, into
        ``request.prompt_token_logprobs`` (None for the first token; its
        prefill skips the prefix cache)."""
        prompt = list(prompt)
        if prompt and (min(prompt) < 0 or max(prompt) >= self.cfg.vocab):
            raise ValueError(f"prompt token ids must lie in [0, {self.cfg.vocab})")
        req = Request(self._next_rid, prompt, max_new_tokens, t_arrive=time.perf_counter(),
                      stop_ids=tuple(int(t) for t in stop_ids), sampling=sampling,
                      logprobs=None if logprobs is None else int(logprobs), prompt_logprobs=bool(prompt_logprobs))
        if sampling is not None and not sampling.greedy and sampling.seed is not None:
            req.rng = torch.Generator(device=self.device)
            req.rng.manual_seed(int(sampling.seed))
        self._next_rid += 1
        self.sched.add(req)
        return req

    def abort(self, rid: int) -> bool:
        """End request ``rid`` between steps (finish_reason "abort"); its KV
        pages and batch slot are freed. Every TP rank must abort the same
        request at the same step."""
        return self.sched.abort(rid)

    def _sync_block_row(self, req):
        row = torch.zeros(self.max_blocks_per_seq, dtype=torch.int32)
        row[: len(req.blocks)] = torch.tensor(req.blocks, dtype=torch.int32)
        # pinned + asynchronous: a pageable copy could stall the host behind the
        # running stream (the host prepares the next chunk meanwhile)
        src = row.pin_memory() if self.device.type == "cuda" else row
        self.block_table[req.slot].copy_(src, non_blocking=True)
        req._row_synced = True

    # ------------------------------------------------------------------ execution
    def _run_prefill(self, batch):
        pieces = batch.pieces
        for p in pieces:
            if not getattr(p.req, "_row_synced", False):
                self._sync_block_row(p.req)
        sampled = any(p.completes and p.req.needs_logits for p in pieces) or \
            any(p.req.prompt_logprobs and not p.decode for p in pieces)
        if self.prefill_graph is not None and len(pieces) == 1 and pieces[0].n == self.chunk and not sampled:
            # a full single-request chunk: replay the captured chunk forward
            p = pieces[0]
            req = p.req
            d = self._h2d(torch.tensor(p.tokens() + list(range(p.start, p.start + p.n)), dtype=torch.int32))
            slots_d = self._h2d(torch.tensor(self.kv.slots(req.blocks, p.start, p.n), dtype=torch.int64))
            return self.prefill_graph.run(d[:p.n], d[p.n:], slots_d, p.start + p.n, self.block_table[req.slot])
        ids, pos, slots, q_lens, kv_lens, rows, last = [], [], [], [], [], [], []
        off = 0
        for p in pieces:
            req = p.req
            ids.extend(p.tokens())
            pos.extend(range(p.start, p.start + p.n))
            slots.extend(self.kv.slots(req.blocks, p.start, p.n))
            q_lens.append(p.n)
            kv_lens.append(p.start + p.n)
            rows.append(req.slot)
            off += p.n
            last.append(off - 1)
        if any(p.req.prompt_logprobs and not p.decode for p in pieces):
            return self._prefill_scoring(pieces, ids, pos, slots, q_lens, kv_lens, rows)
        if sampled:
            hidden = self.forward_prefill(ids, pos, slots, q_lens, kv_lens, rows, last, return_hidden=True)
            return self._sample_tokens(hidden, [p.req for p in pieces], [p.completes for p in pieces])
        return self.forward_prefill(ids, pos, slots, q_lens, kv_lens, rows, last)

    def _prefill_scoring(self, pieces, ids, pos, slots, q_lens, kv_lens, rows):
        """A prefill batch holding a request that scores its prompt: hidden
        states of every row of such pieces (the last row of the others), full
        logits, the prompt tokens' logprobs recorded on their requests, then
        the next token per piece from its last row."""
        want, last_of = [], []
        off = 0
        for p in pieces:
            if p.req.prompt_logprobs and not p.decode:
                want.extend(range(off, off + p.n))
            else:
                want.append(off + p.n - 1)
            last_of.append(len(want) - 1)
            off += p.n
        hidden = self.forward_prefill(ids, pos, slots, q_lens, kv_lens, rows, want, return_hidden=True)
        logits = self.model.full_logits(hidden)
        row = 0
        for p in pieces:
            req = p.req
            if req.prompt_logprobs and not p.decode:
                lp = torch.log_softmax(logits[row:row + p.n].float(), dim=-1)
                if p.start == 0:
                    req.prompt_token_logprobs.append(None)  # the first token has no context
                n_next = min(p.n, len(req.prompt) - 1 - p.start)  # positions whose next token is in the prompt
                if n_next > 0:
                    nxt = torch.tensor(req.prompt[p.start + 1:p.start + 1 + n_next], device=lp.device)
                    vals = lp[:n_next].gather(1, nxt[:, None])[:, 0].tolist()
                    k = req.logprobs or 0
                    if k > 0:
                        tv, ti = torch.topk(lp[:n_next], k, dim=-1)
                        tops = [list(zip(a, b)) for a, b in zip(ti.tolist(), tv.tolist())]
                    else:
                        tops = [[] for _ in vals]
                    req.prompt_token_logprobs.extend(zip(vals, tops))
                row += p.n
            else:
                row += 1
        sel = torch.tensor(last_of, device=logits.device)
        return self._sample_from_logits(logits.index_select(0, sel), [p.req for p in pieces],
                                        [p.completes for p in pieces])

    def forward_prefill(self, ids, pos, slots, q_lens, kv_lens, rows, last, return_hidden=False):
        """One prefill forward from host lists; returns next token per piece
        (or the pieces' final hidden rows with ``return_hidden``)."""
        R = len(q_lens)
        d = self._h2d(torch.tensor(ids + pos + q_lens + kv_lens + rows, dtype=torch.int32))
        T = len(ids)
        ids_d, pos_d = d[:T], d[T:2 * T]
        kvl_d = d[2 * T + R:2 * T + 2 * R]
        rows_d = d[2 * T + 2 * R:2 * T + 3 * R]
        slots_d = self._h2d(torch.tensor(slots, dtype=torch.int64))
        bt = self.block_table.index_select(0, rows_d.long())
        last_d = self._h2d(torch.tensor(last, dtype=torch.int64))
        if self.impl == "oracle":
            def attn(li, q, kc, vc):
                return oracle.paged_attention(q, kc, vc, q_lens, kv_lens, bt)

            return self.model.forward(ids_d, pos_d, slots_d, self.kv.caches, attn, last_d,
                                      return_hidden=return_hidden)
        cu = torch.zeros(R + 1, dtype=torch.int32)
        cu[1:] = torch.tensor(q_lens, dtype=torch.int32).cumsum(0)
        cu_d = self._h2d(cu)
        tiles = self._h2d(ops.prefill_tiles(q_lens))
        scale = self.model.scale
        splits = ops.prefill_splits(tiles.shape[0], self.cfg.heads // self.tp_size, max(kv_lens))

        def attn(li, q, kc, vc):
            return ops.prefill_attention(q, kc, vc, cu_d, kvl_d, bt, tiles, scale, splits=splits)

        halves = self._attn_halves(q_lens, kv_lens, bt, T)
        return self.model.forward(ids_d, pos_d, slots_d, self.kv.caches, attn, last_d, return_hidden=return_hidden,
                                  attn_halves=halves)

    def _attn_halves(self, q_lens, kv_lens, bt, T):
        """Attention of each micro-batch of an overlapped prefill batch
        (model.overlap_split), or None. A piece that straddles the split is
        cut in two: its first rows end the first micro-batch with a kv length
        shortened by the rows that follow; the rest start the second, whose
        keys include the first part (written to the cache earlier in the same
        layer)."""
        T1 = self.model.overlap_split(T)
        if T1 is None:
            return None
        parts = ([], [])  # (q_len, kv_len, piece index) per micro-batch
        start = 0
        for i, (q, kv) in enumerate(zip(q_lens, kv_lens)):
            end = start + q
            if end <= T1:
                parts[0].append((q, kv, i))
            elif start >= T1:
                parts[1].append((q, kv, i))
            else:
                n0 = T1 - start
                parts[0].append((n0, kv - (q - n0), i))
                parts[1].append((q - n0, kv, i))
            start = end
        scale = self.model.scale
        nq = self.cfg.heads // self.tp_size
        fns = []
        for pl in parts:
            ql = [p[0] for p in pl]
            kl = [p[1] for p in pl]
            cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
            cu[1:] = torch.tensor(ql, dtype=torch.int32).cumsum(0)
            meta = self._h2d(torch.cat([cu, torch.tensor(kl, dtype=torch.int32),
                                        torch.tensor([p[2] for p in pl], dtype=torch.int32)]))
            n = len(ql)
            cu_h, kvl_h, sel = meta[:n + 1], meta[n + 1:2 * n + 1], meta[2 * n + 1:]
            bt_h = bt.index_select(0, sel.long())
            tiles_h = self._h2d(ops.prefill_tiles(ql))
            splits_h = ops.prefill_splits(tiles_h.shape[0], nq, max(kl))

            def f(li, q, kc, vc, cu_h=cu_h, kvl_h=kvl_h, bt_h=bt_h, tiles_h=tiles_h, splits_h=splits_h):
                return ops.prefill_attention(q, kc, vc, cu_h, kvl_h, bt_h, tiles_h, scale, splits=splits_h)
            fns.append(f)
        return (T1, fns[0], fns[1])

    def decode_inputs(self, reqs):
        """(last token, position, kv length, cache slot, table row) per request."""
        ids, pos, kv_len, slots, rows = [], [], [], [], []
        for r in reqs:  # one pass: this runs every decode step
            out = r.output
            n = len(r.prompt) + len(out)
            ids.append(out[-1] if out else r.prompt[-1])
            pos.append(n - 1)
            kv_len.append(n)
            slots.append(r.blocks[(n - 1) // PAGE] * PAGE + (n - 1) % PAGE)
            rows.append(r.slot)
        return ids, pos, kv_len, slots, rows

    def forward_decode_eager(self, ids_d, pos_d, kvl_d, slots_d, rows_d, splits=None, return_hidden=False):
        B = ids_d.shape[0]
        bt = self.block_table.index_select(0, rows_d.long())
        if self.impl == "oracle":
            kv_lens = kvl_d.tolist()

            def attn(li, q, kc, vc):
                return oracle.paged_attention(q, kc, vc, [1] * B, kv_lens, bt)
        else:
            nkv = self.cfg.kv_heads // self.tp_size
            sp = splits or ops.decode_splits(B, nkv, self.max_seq)
            scale = self.model.scale

            def attn(li, q, kc, vc):
                return ops.decode_attention(q, kc, vc, kvl_d, bt, scale, splits=sp)

        last = torch.arange(B, device=self.device, dtype=torch.int64)
        return self.model.forward(ids_d, pos_d, slots_d, self.kv.caches, attn, last, return_hidden=return_hidden)

    def _run_decode(self, batch):
        for r in batch.reqs:
            if not getattr(r, "_row_synced", False):
                self._sync_block_row(r)
        ids, pos, kv_len, slots, rows = self.decode_inputs(batch.reqs)
        sampled = any(r.needs_logits for r in batch.reqs)
        if self.graphs is not None and self.graphs.can_run(len(ids)):
            if not sampled:
                return self.graphs.run(ids, pos, kv_len, slots, rows)
            if self.sample_in_graphs:
                logits = self.graphs.run_logits(ids, pos, kv_len, slots, rows)
                return self._sample_from_logits(logits, batch.reqs)
        B = len(ids)
        d = self._h2d(torch.tensor(ids + pos + kv_len + rows, dtype=torch.int32))
        slots_d = self._h2d(torch.tensor(slots, dtype=torch.int64))
        if sampled:
            hidden = self.forward_decode_eager(d[:B], d[B:2 * B], d[2 * B:3 * B], slots_d, d[3 * B:],
                                               return_hidden=True)
            return self._sample_tokens(hidden, batch.reqs)
        return self.forward_decode_eager(d[:B], d[B:2 * B], d[2 * B:3 * B], slots_d, d[3 * B:])

    def step(self):
        """Run one scheduled batch; returns the batch (or None when idle)."""
        batch = self.sched.next_batch()
        if batch is None:
            return None
        with nvtx.rng(f"{batch.kind} tokens={batch.num_tokens}"):
            return self._step(batch)

    def _step(self, batch):
        if batch.kind == "prefill":
            out = self._run_prefill(batch)
            if any(p.completes for p in batch.pieces):
                nxt = out.tolist()
            else:
                # no prompt ends in this chunk, so no token is used: skip the
                # device->host read (a sync), and the host prepares the next
                # chunk while this one runs
                nxt = [0] * len(batch.pieces)
            now = time.perf_counter()
            for p in batch.pieces:
                if p.completes:
                    if not p.decode:
                        p.req.t_first = now
                    p.req.token_times.append(now)
            self.sched.after_prefill(batch, nxt)
        else:
            nxt = self._run_decode(batch).tolist()
            now = time.perf_counter()
            for r in batch.reqs:
                r.token_times.append(now)
            self.sched.after_decode(batch, nxt)
        return batch

    def run(self):
        while self.sched.has_work():
            self.step()
        done = sorted(self.sched.finished, key=lambda r: r.rid)
        self.sched.finished = []
        return done

    def generate(self, prompts, max_new_tokens: int = 16, stop_ids=(), sampling=None):
        reqs = [self.add_request(p, max_new_tokens, stop_ids, sampling) for p in prompts]
        self.run()
        return [r.output for r in reqs]

    def generate_text(self, prompts, sampling_params: dict = None, return_logprob: bool = False,
                      top_logprobs_num: int = 0):
        """Offline generation over text, in the shape of sglang's offline
        engine: ``prompts`` is a string or a list of strings;
        ``sampling_params`` a dict of ``max_new_tokens`` (16), ``temperature``
        (0: greedy), ``top_k``, ``top_p``, ``seed``, ``stop_token_ids``
        (default: the checkpoint's EOS ids), ``presence_penalty``,
        ``frequency_penalty``, ``repetition_penalty``, ``logit_bias`` ({id:
        bias}), ``min_new_tokens``, ``ignore_eos`` (generate past the
        checkpoint's EOS ids) and ``stop`` (a string or a list: the
        request ends once its text holds one, and the text and token ids are
        cut before it, finish reason "stop"). Returns one ``{"text",
        "token_ids", "finish_reason", "meta_info"}`` per prompt (a single dict
        for a single string); ``meta_info`` is sglang's (prompt and
        completion token counts, ``finish_reason: {"type": ...}``). ``return_logprob`` adds ``"logprobs"``: per generated token
        (id, logprob, [(id, logprob)] of the ``top_logprobs_num`` most likely)."""
        from .stops import find_stop, stop_prefix, tail_hit
        from .tokenizer import ByteTokenizer

        tok = self.tokenizer or ByteTokenizer()
        sp = dict(sampling_params or {})
        max_new = int(sp.pop("max_new_tokens", 16))
        stop = sp.pop("stop_token_ids", None)
        ignore_eos = bool(sp.pop("ignore_eos", False))
        stop = (() if ignore_eos else self.default_stop_ids) if stop is None else tuple(stop)
        stop_strs = sp.pop("stop", None) or ()
        stop_strs = tuple(x for x in ((stop_strs,) if isinstance(stop_strs, str) else stop_strs) if x)
        temp = float(sp.pop("temperature", 0.0))
        top_k, top_p, seed = int(sp.pop("top_k", 0)), float(sp.pop("top_p", 1.0)), sp.pop("seed", None)
        adj = dict(presence_penalty=float(sp.pop("presence_penalty", 0.0)),
                   frequency_penalty=float(sp.pop("frequency_penalty", 0.0)),
                   repetition_penalty=float(sp.pop("repetition_penalty", 1.0)),
                   logit_bias=tuple(sorted((int(k), float(v)) for k, v in dict(sp.pop("logit_bias", {})).items())),
                   min_new_tokens=int(sp.pop("min_new_tokens", 0)))
        if sp:
            raise ValueError(f"unknown sampling params: {', '.join(sorted(sp))}")
        sampling = SamplingParams(max(temp, 0.0), top_k, top_p, seed, **adj)
        if not sampling.adjusts and temp <= 0:
            sampling = None
        single = isinstance(prompts, str)
        lp = int(top_logprobs_num) if return_logprob else None
        reqs = [self.add_request(tok.encode(p), max_new, stop, sampling, logprobs=lp)
                for p in ([prompts] if single else prompts)]
        if stop_strs:
            # the same check on every TP rank (same tokens, same tokenizer), so
            # every rank aborts a request at the same step
            checked = {r.rid: 0 for r in reqs}
            while self.sched.has_work():
                self.step()
                for r in reqs:
                    if r.finish_reason is None and len(r.output) > checked[r.rid]:
                        checked[r.rid] = len(r.output)
                        if tail_hit(r.output, stop_strs, tok.decode):
                            self.abort(r.rid)
            self.sched.finished = []
        else:
            self.run()
        out = []
        for r in reqs:
            ids, reason = list(r.output), r.finish_reason
            text = tok.decode(ids)
            if stop_strs:
                k = stop_prefix(ids, stop_strs, tok.decode)
                if k is not None:
                    ids, reason = ids[:k], "stop"
                    text = tok.decode(ids)
                    text = text[:find_stop(text, stop_strs)]
            o = {"text": text, "token_ids": ids, "finish_reason": reason,
                 "meta_info": {"prompt_tokens": len(r.prompt), "completion_tokens": len(ids),
                               "finish_reason": {"type": reason}}}
            if return_logprob:
                o["logprobs"] = [(t, c, top) for t, (c, top) in zip(ids, r.token_logprobs)]
            out.append(o)
        return out[0] if single else out
