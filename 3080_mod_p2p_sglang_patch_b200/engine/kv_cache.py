"""Paged KV cache (page = 16 tokens, bf16) and its block allocator.

Layout per layer: k, v = [num_blocks, kv_heads_per_rank, 16, head_dim] - one
contiguous 4 KB page per (block, kv head), the unit the attention kernels
stream. Block 0 is reserved as a scratch page for padded decode rows.
(The reference relies on sglang's paged cache; it ships none.)
"""
import numpy as np
import torch

PAGE = 16


class BlockAllocator:
    def __init__(self, num_blocks: int, reserved: int = 1):
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, reserved - 1, -1))

    @property
    def free(self) -> int:
        return len(self._free)

    def alloc(self, n: int):
        if n > len(self._free):
            raise MemoryError(f"KV cache out of blocks: need {n}, have {len(self._free)}")
        out = [self._free.pop() for _ in range(n)]
        return out

    def release(self, blocks):
        self._free.extend(reversed(blocks))


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

    def slots(self, blocks, start: int, n: int):
        """Cache slots (block*PAGE + offset) of token positions [start, start+n)."""
        if n <= 0:
            return []
        pos = np.arange(start, start + n, dtype=np.int64)
        return (np.asarray(blocks, dtype=np.int64)[pos // PAGE] * PAGE + pos % PAGE).tolist()
