"""Paged KV cache (page = 16 tokens, bf16) and its block allocator.

Layout per layer: k, v = [num_blocks, kv_heads_per_rank, 16, head_dim] - one
contiguous 4 KB page per (block, kv head), the unit the attention kernels
stream. Block 0 is reserved as a scratch page for padded decode rows.
(The reference relies on sglang's paged cache; it ships none.)
"""
import collections

import numpy as np
import torch

PAGE = 16


class BlockAllocator:
    def __init__(self, num_blocks: int, reserved: int = 1):
        self.num_blocks = num_blocks
        self.reserved = reserved
        self._free = list(range(num_blocks - 1, reserved - 1, -1))

    @property
    def free(self) -> int:
        return len(self._free)

    @property
    def capacity(self) -> int:
        """Blocks that can ever be handed out (all but the reserved ones)."""
        return self.num_blocks - self.reserved

    def alloc(self, n: int):
        if n > len(self._free):
            raise MemoryError(f"KV cache out of blocks: need {n}, have {len(self._free)}")
        out = [self._free.pop() for _ in range(n)]
        return out

    def release(self, blocks):
        self._free.extend(reversed(blocks))


class PrefixCache:
    """Shared full KV pages of prompt prefixes (the role of sglang's radix
    cache, at page granularity).

    A full page of prompt tokens is keyed by the chain (key of the previous
    page, its 16 token ids), so a key names one exact prefix; the stored
    tokens are compared on a hit. Pages are registered when the request that
    computed them finishes its prefill, and carry a reference count: a new
    request whose prompt starts with cached pages takes references and
    prefills only the rest. Unreferenced pages stay cached in LRU order and
    are evicted when the allocator runs short. Cached pages are never written
    again: a request's own writes start after its matched pages.
    """

    def __init__(self, allocator: BlockAllocator):
        self.alloc = allocator
        self.table = {}     # chain hash -> (block, page tokens)
        self.key_of = {}    # block -> key
        self.ref = {}       # cached block -> references from live requests
        self.lru = collections.OrderedDict()  # unreferenced cached blocks, oldest first
        self.hits = 0       # pages served from the cache

    @staticmethod
    def page_keys(tokens, pages: int):
        keys, prev = [], None
        for i in range(pages):
            page = tuple(tokens[i * PAGE:(i + 1) * PAGE])
            prev = hash((prev, page))
            keys.append((prev, page))
        return keys

    @property
    def evictable(self) -> int:
        return len(self.lru)

    def match(self, tokens, max_pages: int):
        """Cached blocks of the longest run of leading full pages (<= max_pages)."""
        out = []
        for key, page in self.page_keys(tokens, max_pages):
            hit = self.table.get(key)
            if hit is None or hit[1] != page:
                break
            out.append(hit[0])
        return out

    def acquire(self, blocks):
        for b in blocks:
            if self.ref[b] == 0:
                self.lru.pop(b, None)
            self.ref[b] += 1
        self.hits += len(blocks)

    def flush(self) -> int:
        """Evict every unreferenced cached page (sglang's flush_cache); pages
        live requests hold stay. Returns the pages freed."""
        n = 0
        while self.lru:
            b, _ = self.lru.popitem(last=False)
            del self.table[self.key_of.pop(b)]
            del self.ref[b]
            self.alloc.release([b])
            n += 1
        return n

    def alloc_blocks(self, n: int):
        """n free blocks, evicting unreferenced cached pages (oldest first) if needed."""
        while self.alloc.free < n and self.lru:
            b, _ = self.lru.popitem(last=False)
            del self.table[self.key_of.pop(b)]
            del self.ref[b]
            self.alloc.release([b])
        return self.alloc.alloc(n)

    def insert(self, tokens, blocks, first_page: int, pages: int):
        """Register pages [first_page, pages) of a request's prompt (computed
        into ``blocks``); the request keeps one reference to each."""
        keys = self.page_keys(tokens, pages)
        for i in range(first_page, pages):
            key, page = keys[i]
            if key in self.table:  # computed concurrently by another request: keep ours private
                continue
            b = blocks[i]
            self.table[key] = (b, page)
            self.key_of[b] = key
            self.ref[b] = 1

    def release(self, blocks):
        """A finished request's blocks: cached ones lose a reference (and become
        evictable at zero), private ones go back to the allocator."""
        private = []
        for b in blocks:
            if b in self.ref:
                self.ref[b] -= 1
                if self.ref[b] == 0:
                    self.lru[b] = None
            else:
                private.append(b)
        if private:
            self.alloc.release(private)


class PagedKVCache:
    def __init__(self, layers: int, kv_heads: int, head_dim: int, num_blocks: int, device, dtype=torch.bfloat16):
        self.layers = layers
        self.num_blocks = num_blocks
        self.storage = torch.zeros((layers, 2, num_blocks, kv_heads, PAGE, head_dim), dtype=dtype, device=device)
        self.caches = [(self.storage[l, 0], self.storage[l, 1]) for l in range(layers)]
        self.alloc = BlockAllocator(num_blocks)

    @staticmethod
    def blocks_for(tokens: int) -> int:
        return (tokens + PAGE - 1) // PAGE

    @staticmethod
    def bytes_per_token(layers, kv_heads, head_dim, dtype_bytes=2):
        return layers * 2 * kv_heads * head_dim * dtype_bytes

    @staticmethod
    def blocks_for_memory(total_bytes: int, free_bytes: int, fraction: float, block_bytes: int) -> int:
        """Blocks that fit when weights plus KV cache may use ``fraction`` of
        the device's memory (sglang's ``--mem-fraction-static``): the budget
        is fraction x total minus what is already in use."""
        budget = fraction * total_bytes - (total_bytes - free_bytes)
        return max(0, int(budget // block_bytes))

    def slots(self, blocks, start: int, n: int):
        """Cache slots (block*PAGE + offset) of token positions [start, start+n)."""
        if n <= 0:
            return []
        pos = np.arange(start, start + n, dtype=np.int64)
        return (np.asarray(blocks, dtype=np.int64)[pos // PAGE] * PAGE + pos % PAGE).tolist()
