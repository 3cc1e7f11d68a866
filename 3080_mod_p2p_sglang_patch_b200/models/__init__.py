"""Model family: Llama-style dense decoder with tensor parallelism."""
from .config import LlamaConfig  # noqa: F401
from .llama import LlamaTP, LlamaWeights  # noqa: F401
