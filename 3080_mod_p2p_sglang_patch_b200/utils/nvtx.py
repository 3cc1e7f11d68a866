"""NVTX ranges around engine steps and decoder layers, for timeline tools
(Nsight Systems and the like). Off unless ``MBX_NVTX=1``: then every
``rng(name)`` pushes a range on the CUDA profiler's NVTX stack; otherwise it
is an empty context manager. Ranges are host markers, so inside a captured
CUDA graph they appear at capture time only."""
import contextlib
import os

ENABLED = os.environ.get("MBX_NVTX", "0") == "1"


@contextlib.contextmanager
def _range(name):
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


_NULL = contextlib.nullcontext()


def rng(name: str):
    return _range(name) if ENABLED else _NULL
