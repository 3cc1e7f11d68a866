"""OpenAI-compatible HTTP front end for the TP engine (the role of sglang's
``launch_server`` in the reference's flow: ``SGLANG_MAILBOX_AR=1 ...
launch_server --tp 2``, reference scripts/sglang-p2p.sh:162; its
prompt-processing bench posts to ``/v1/chat/completions`` and reads
``usage.prompt_tokens``, tests/pp_bench.py:21-29).

    SGLANG_MAILBOX_AR=1 python -m 3080_mod_p2p_sglang_patch_b200.server --model /path/to/ckpt --tp 2
    torchrun --nproc-per-node N -m 3080_mod_p2p_sglang_patch_b200.server --model 8b --port 8001

One process per GPU. ``--tp N`` outside torchrun starts the N ranks itself
(torch.distributed.run on 127.0.0.1); under torchrun the ranks are
torchrun's. sglang's spellings of the common flags are accepted
(``--tp-size``, ``--chunked-prefill-size``, ``--context-length``,
``--max-running-requests``, ``--disable-cuda-graph``).

Rank 0 serves HTTP and owns the request queue; every rank runs the same
engine loop in lockstep: at each iteration rank 0 broadcasts the newly
arrived requests over a gloo control group, every rank adds them in the same
order and runs one engine step (the TP collectives of that step then line up
across ranks). With ``SGLANG_MAILBOX_AR=1`` the TP allreduces go through
MailboxAR, otherwise NCCL.

``--model DIR`` (or ``--model-path DIR``) serves a Hugging Face checkpoint
(safetensors, each rank reads its shards) with the directory's tokenizer
(through transformers, local files only) and its chat template. ``--model
8b|70b|tiny`` runs random weights, and text goes through a byte tokenizer:
UTF-8 bytes are token ids 0..255, generated ids >= 256 decode to nothing.
Token-id prompts (``"prompt": [ids]``) are accepted either way. Decoding is
greedy unless a request sets ``temperature`` (with ``top_p``, ``top_k``,
``seed``).
"""
from ..engine.tokenizer import ByteTokenizer, HFTokenizer, load_chat_template  # noqa: F401
from .cli import (RANDOM_MODELS, build_parser, main, relaunch_command, replica_commands,  # noqa: F401
                  resolve_model)
from .http import build_app, render_metrics, start_http  # noqa: F401
from .loop import EngineServer, Overloaded, _Pending  # noqa: F401
