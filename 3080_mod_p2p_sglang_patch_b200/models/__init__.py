"""Model family: Llama-style dense decoder with tensor parallelism (random-init
or loaded from Hugging Face safetensors checkpoints)."""
from .config import LlamaConfig  # noqa: F401
from .llama import LlamaTP, LlamaWeights  # noqa: F401
from .loader import SafeTensors, config_from_hf, load_llama, stop_token_ids, write_safetensors  # noqa: F401
