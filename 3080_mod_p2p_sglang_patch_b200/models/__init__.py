"""Model family: Llama-style dense decoder with tensor parallelism (random-init
or loaded from Hugging Face safetensors checkpoints)."""
from .config import LlamaConfig  # noqa: F401
from .llama import LlamaTP, LlamaWeights  # noqa: F401
from .loader import (SafeTensors, awq_dequant, awq_pack, awq_quantize, awq_unpack, config_from_hf,  # noqa: F401
                     load_llama, quantize_weights_int4, stop_token_ids, write_safetensors)
