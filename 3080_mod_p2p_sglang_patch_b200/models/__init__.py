"""Model family: Llama-style dense decoder with tensor parallelism (random-init
or loaded from Hugging Face safetensors checkpoints)."""
from .config import LlamaConfig  # noqa: F401
from .llama import LlamaTP, LlamaWeights  # noqa: F401
from .loader import (SafeTensors, awq_dequant, awq_pack, awq_quantize, awq_unpack, config_from_hf,  # noqa: F401
                     config_to_hf, load_llama, quantize_weights_int4, save_llama, stop_token_ids,
                     write_safetensors)
