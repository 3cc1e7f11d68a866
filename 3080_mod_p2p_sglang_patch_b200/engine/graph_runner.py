"""CUDA-graph decode runner for fixed batch sizes (default {1, 8, 32, 64}).

Decode steps are launch-bound (2 collectives + ~10 kernels per layer), so
each batch size's whole forward - embedding, every layer's GEMMs, attention,
fused allreduce+RMSNorm collectives, LM head and the vocab-parallel argmax -
is captured once and replayed. Inputs are copied into static buffers with one
pinned host->device copy; padded rows decode into a reserved scratch page.
The communicator's buffers and epochs never move, so replays need no
re-registration (the reference's graph story, docs/principle.md:80-83).
"""
import torch

from .. import ops
from .kv_cache import PAGE


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
        self.graphs = {}
        self.outputs = {}
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

    def capture(self):
        e = self.e
        nkv = e.cfg.kv_heads // e.tp_size
        # padded rows: position 0, kv_len 1, slot in the reserved block 0, table row 0
        self.in_i32.zero_()
        self.in_i32[2 * self.max_bs:3 * self.max_bs].fill_(1)
        self.in_slots.zero_()
        torch.cuda.synchronize()
        s = torch.cuda.Stream(device=e.device)
        s.wait_stream(torch.cuda.current_stream(e.device))
        with torch.cuda.stream(s):
            for bs in reversed(self.sizes):
                ids, pos, kvl, slots, rows = self._views(bs)
                splits = ops.decode_splits(bs, nkv, e.max_seq)
                for _ in range(2):  # warm-up (tensor maps, lazy init)
                    e.forward_decode_eager(ids, pos, kvl, slots, rows, splits=splits)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                comm = e.tp.ca_comm if e.tp is not None else None
                ctx = comm.capture() if comm is not None else _null()
                with ctx:
                    with torch.cuda.graph(g, pool=self.pool, stream=s):
                        out = e.forward_decode_eager(ids, pos, kvl, slots, rows, splits=splits)
                if self.pool is None:
                    self.pool = g.pool()
                self.graphs[bs] = g
                self.outputs[bs] = out
        torch.cuda.current_stream(e.device).wait_stream(s)
        torch.cuda.synchronize()
        self._captured = True

    def run(self, ids, pos, kv_len, slots, rows):
        if not self._captured:
            self.capture()
        B = len(ids)
        bs = next(s for s in self.sizes if s >= B)
        n = self.max_bs
        h = self.host_i32
        pad = bs - B
        h[0:bs] = torch.tensor(ids + [0] * pad, dtype=torch.int32)
        h[n:n + bs] = torch.tensor(pos + [0] * pad, dtype=torch.int32)
        h[2 * n:2 * n + bs] = torch.tensor(kv_len + [1] * pad, dtype=torch.int32)
        h[3 * n:3 * n + bs] = torch.tensor(rows + [0] * pad, dtype=torch.int32)
        self.host_slots[:bs] = torch.tensor(slots + [0] * pad, dtype=torch.int64)
        self.in_i32.copy_(h, non_blocking=True)
        self.in_slots.copy_(self.host_slots, non_blocking=True)
        self.graphs[bs].replay()
        return self.outputs[bs][:B]

    def close(self):
        self.graphs.clear()
        self.outputs.clear()


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
