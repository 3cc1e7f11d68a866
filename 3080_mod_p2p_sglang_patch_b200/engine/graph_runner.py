"""CUDA-graph decode runner for fixed batch sizes (default {1, 8, 32, 64}).

Decode steps are launch-bound (2 collectives + ~10 kernels per layer), so
each batch size's whole forward - embedding, every layer's GEMMs, attention,
fused allreduce+RMSNorm collectives, LM head and the vocab-parallel argmax -
is captured once and replayed. Inputs are copied into static buffers with one
pinned host->device copy; padded rows decode into a reserved scratch page.
The communicator's buffers and epochs never move, so replays need no
re-registration (the reference's graph story, docs/principle.md:80-83).
"""
import contextlib
import gc

import torch

from .. import ops
from ..utils import launches


@contextlib.contextmanager
def no_gc():
    """Collect garbage, then keep the collector off for the capture.

    A capture in the global mode is invalidated by a graph or other CUDA
    resource destroyed meanwhile, and the collector runs whenever allocations
    pile up: an unreachable engine of an earlier caller freeing its captured
    graphs in the middle of this capture ends it with
    ``cudaErrorStreamCaptureInvalidated``."""
    gc.collect()
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()


class DecodeGraphRunner:
    def __init__(self, engine, sizes=(1, 8, 32, 64)):
        self.e = engine
        self.sizes = tuple(sorted(sizes))
        self.max_bs = self.sizes[-1] if self.sizes else 0
        dev = engine.device
        n = self.max_bs
        # packed int32 inputs: ids | pos | kv_len | rows ; slots separately (int64)
        self.in_i32 = torch.zeros(4 * n, dtype=torch.int32, device=dev)
        self.in_slots = torch.zeros(n, dtype=torch.int64, device=dev)
        self.host_i32 = torch.zeros(4 * n, dtype=torch.int32).pin_memory()
        self.host_slots = torch.zeros(n, dtype=torch.int64).pin_memory()
        # completion of the last host->device copy out of the pinned buffers:
        # they are rewritten only after it (copies are asynchronous)
        self._copied = None
        self.graphs = {}
        self.outputs = {}
        self.kernels = {}
        # graphs that end in the full logits (sampled / logprob batches), per
        # batch size, captured on first use
        self.logit_graphs = {}
        self.logit_outputs = {}
        self.pool = None
        self._captured = False

    def can_run(self, bs):
        return bs <= self.max_bs

    def _views(self, bs):
        n = self.max_bs
        ids = self.in_i32[0:bs]
        pos = self.in_i32[n:n + bs]
        kvl = self.in_i32[2 * n:2 * n + bs]
        rows = self.in_i32[3 * n:3 * n + bs]
        return ids, pos, kvl, self.in_slots[:bs], rows

    def _capture_sizes(self, sizes, logits: bool):
        """Capture one graph per batch size: the decode forward ending in the
        next tokens (greedy), or with ``logits`` in the full fp32 logits.
        Collective on the TP ranks (warm-ups and capture run collectives)."""
        e = self.e
        nkv = e.cfg.kv_heads // e.tp_size
        # padded rows: position 0, kv_len 1, slot in the reserved block 0, table row 0
        self.in_i32.zero_()
        self.in_i32[2 * self.max_bs:3 * self.max_bs].fill_(1)
        self.in_slots.zero_()
        torch.cuda.synchronize()

        def fwd(ids, pos, kvl, slots, rows, splits):
            if not logits:
                return e.forward_decode_eager(ids, pos, kvl, slots, rows, splits=splits)
            hidden = e.forward_decode_eager(ids, pos, kvl, slots, rows, splits=splits, return_hidden=True)
            return e.model.full_logits(hidden)

        s = torch.cuda.Stream(device=e.device)
        s.wait_stream(torch.cuda.current_stream(e.device))
        with torch.cuda.stream(s):
            for bs in reversed(sizes):
                ids, pos, kvl, slots, rows = self._views(bs)
                splits = ops.decode_splits(bs, nkv, e.max_seq)
                for _ in range(2):  # warm-up (tensor maps, lazy init)
                    fwd(ids, pos, kvl, slots, rows, splits)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                comm = e.tp.ca_comm if e.tp is not None else None
                ctx = comm.capture() if comm is not None else _null()
                before = launches.get()
                with ctx, no_gc():
                    with torch.cuda.graph(g, pool=self.pool, stream=s):
                        out = fwd(ids, pos, kvl, slots, rows, splits)
                n_kernels = launches.get() - before
                if self.pool is None:
                    self.pool = g.pool()
                if logits:
                    self.logit_graphs[bs], self.logit_outputs[bs] = g, out
                    self.kernels[("logits", bs)] = n_kernels
                else:
                    self.graphs[bs], self.outputs[bs] = g, out
                    self.kernels[bs] = n_kernels
        torch.cuda.current_stream(e.device).wait_stream(s)
        torch.cuda.synchronize()

    def capture(self):
        self._capture_sizes(self.sizes, logits=False)
        self._captured = True

    def run(self, ids, pos, kv_len, slots, rows):
        if not self._captured:
            self.capture()
        return self._replay(ids, pos, kv_len, slots, rows, logits=False)

    def run_logits(self, ids, pos, kv_len, slots, rows):
        """Replay the graph that ends in the full fp32 logits [B, V] (every
        TP rank gets the same values), capturing it for this batch size on
        first use."""
        if not self._captured:
            self.capture()
        bs = next(s for s in self.sizes if s >= len(ids))
        if bs not in self.logit_graphs:
            self._capture_sizes((bs,), logits=True)
        return self._replay(ids, pos, kv_len, slots, rows, logits=True)

    def _replay(self, ids, pos, kv_len, slots, rows, logits):
        B = len(ids)
        bs = next(s for s in self.sizes if s >= B)
        n = self.max_bs
        h = self.host_i32
        pad = bs - B
        if self._copied is not None:
            self._copied.synchronize()
        h[0:bs] = torch.tensor(ids + [0] * pad, dtype=torch.int32)
        h[n:n + bs] = torch.tensor(pos + [0] * pad, dtype=torch.int32)
        h[2 * n:2 * n + bs] = torch.tensor(kv_len + [1] * pad, dtype=torch.int32)
        h[3 * n:3 * n + bs] = torch.tensor(rows + [0] * pad, dtype=torch.int32)
        self.host_slots[:bs] = torch.tensor(slots + [0] * pad, dtype=torch.int64)
        self.in_i32.copy_(h, non_blocking=True)
        self.in_slots.copy_(self.host_slots, non_blocking=True)
        if self._copied is None:
            self._copied = torch.cuda.Event()
        self._copied.record()
        if logits:
            self.logit_graphs[bs].replay()
            launches.add(self.kernels.get(("logits", bs), 0))
            return self.logit_outputs[bs][:B]
        self.graphs[bs].replay()
        launches.add(self.kernels.get(bs, 0))
        return self.outputs[bs][:B]

    def close(self):
        self.graphs.clear()
        self.outputs.clear()
        self.logit_graphs.clear()
        self.logit_outputs.clear()


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class PrefillGraphRunner:
    """CUDA graph of one full prefill chunk (one request, T = chunk tokens).

    At high TP a chunk's GPU work per rank is smaller than the host time to
    launch its ~700 kernels one by one, so the whole chunk forward is captured
    once and replayed with its inputs in static device buffers: token ids,
    positions, cache slots, the request's kv length and block-table row. The
    query-tile list and the split-KV factor are fixed at capture (the kernel
    derives the causal bounds from the kv length at run time).
    """

    def __init__(self, engine, T: int):
        self.e = engine
        self.T = T
        dev = engine.device
        self.ids = torch.zeros(T, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(T, dtype=torch.int32, device=dev)
        self.slots = torch.zeros(T, dtype=torch.int64, device=dev)
        self.kvl = torch.full((1,), T, dtype=torch.int32, device=dev)
        self.cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
        self.bt = torch.zeros((1, engine.max_blocks_per_seq), dtype=torch.int32, device=dev)
        self.tiles = ops.prefill_tiles([T]).to(dev)
        self.last = torch.tensor([T - 1], dtype=torch.int64, device=dev)
        nq = engine.cfg.heads // engine.tp_size
        self.splits = ops.prefill_splits(self.tiles.shape[0], nq, engine.max_seq)
        ops.workspace(dev).prefill(T * nq * self.splits * 128, T * nq * self.splits)
        # overlapped micro-batches (model.enable_overlap): rows [0, T1) and
        # [T1, T) of the chunk, each with its own attention metadata; the
        # first half's kv length is the chunk's minus T - T1
        self.T1 = engine.model.overlap_split(T)
        self.halves = None
        if self.T1 is not None:
            self.halves = []
            for n in (self.T1, T - self.T1):
                tiles = ops.prefill_tiles([n]).to(dev)
                splits = ops.prefill_splits(tiles.shape[0], nq, engine.max_seq)
                ops.workspace(dev).prefill(n * nq * splits * 128, n * nq * splits)
                self.halves.append({"cu": torch.tensor([0, n], dtype=torch.int32, device=dev), "tiles": tiles,
                                    "splits": splits, "kvl": torch.full((1,), n, dtype=torch.int32, device=dev)})
            self.halves[1]["kvl"] = self.kvl
        self.graph = None
        self.out = None

    def _forward(self):
        e = self.e
        scale = e.model.scale

        def attn(li, q, kc, vc):
            return ops.prefill_attention(q, kc, vc, self.cu, self.kvl, self.bt, self.tiles, scale, splits=self.splits)

        halves = None
        if self.halves is not None:
            def half_attn(h):
                def f(li, q, kc, vc):
                    return ops.prefill_attention(q, kc, vc, h["cu"], h["kvl"], self.bt, h["tiles"], scale,
                                                 splits=h["splits"])
                return f
            halves = (self.T1, half_attn(self.halves[0]), half_attn(self.halves[1]))
        return e.model.forward(self.ids, self.pos, self.slots, e.kv.caches, attn, self.last, attn_halves=halves)

    def capture(self):
        e = self.e
        # warm-up on the scratch block 0 (slots 0..T-1 of block 0.. would clobber
        # real pages, so point every slot at the reserved block's first entry)
        self.slots.zero_()
        self.pos.copy_(torch.arange(self.T, dtype=torch.int32, device=e.device))
        self.kvl.fill_(self.T)
        if self.halves is not None:
            self.halves[0]["kvl"].fill_(self.T1)
        torch.cuda.synchronize()
        s = torch.cuda.Stream(device=e.device)
        s.wait_stream(torch.cuda.current_stream(e.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._forward()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            comm = e.tp.ca_comm if e.tp is not None else None
            ctx = comm.capture() if comm is not None else _null()
            before = launches.get()
            with ctx, no_gc():
                with torch.cuda.graph(g, stream=s):
                    self.out = self._forward()
            self.kernels_per_replay = launches.get() - before
        torch.cuda.current_stream(e.device).wait_stream(s)
        torch.cuda.synchronize()
        self.graph = g

    def run(self, ids_d, pos_d, slots_d, kv_len: int, bt_row_d):
        """Device tensors in, next token (int64 [1]) out."""
        if self.graph is None:
            self.capture()
        self.ids.copy_(ids_d, non_blocking=True)
        self.pos.copy_(pos_d, non_blocking=True)
        self.slots.copy_(slots_d, non_blocking=True)
        self.kvl.fill_(kv_len)
        if self.halves is not None:
            self.halves[0]["kvl"].fill_(kv_len - (self.T - self.T1))
        self.bt.copy_(bt_row_d.view(1, -1), non_blocking=True)
        self.graph.replay()
        launches.add(self.kernels_per_replay)
        return self.out

    def close(self):
        self.graph = None
        self.out = None
