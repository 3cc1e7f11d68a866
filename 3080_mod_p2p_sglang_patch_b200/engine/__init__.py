"""Serving engine: paged KV cache, chunked-prefill scheduler, CUDA-graph
decode runner, offline LLM engine."""
from .engine import LLMEngine  # noqa: F401
from .graph_runner import DecodeGraphRunner  # noqa: F401
from .kv_cache import PAGE, BlockAllocator, PagedKVCache, PrefixCache  # noqa: F401
from .sampling import SamplingParams, sample  # noqa: F401
from .scheduler import Batch, PrefillPiece, Request, Scheduler  # noqa: F401
