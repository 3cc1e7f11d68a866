"""B200-native tensor-parallel allreduce communicator + sglang-style TP engine.

The package name starts with a digit, so import it with importlib::

    import importlib
    mbx = importlib.import_module("3080_mod_p2p_sglang_patch_b200")
    MailboxAR = mbx.parallel.MailboxAR

Subpackages: ``parallel`` (symmetric memory, MailboxAR communicator, TP groups,
sglang dispatch hook), ``ops`` (sm_100a kernels: tcgen05 GEMM, attention,
norms, RoPE, activation, sampling), ``models`` (Llama-style TP decoder),
``engine`` (paged KV cache, chunked-prefill scheduler, CUDA-graph decode
runner, offline LLM engine), ``utils`` (timing, clocks, preflight).
"""
from . import config  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # Lazy subpackage import keeps `import` cheap (no CUDA work at import time).
    import importlib

    if name in ("parallel", "ops", "models", "engine", "utils"):
        mod = importlib.import_module(f".{name}", __name__)
        globals()[name] = mod
        return mod
    raise AttributeError(name)
