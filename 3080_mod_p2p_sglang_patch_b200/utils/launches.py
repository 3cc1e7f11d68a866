"""Count of this package's kernel launches (for the bench's gpu_launches).

Every op wrapper and communicator call adds the number of kernels it
launches; CUDA-graph replays add the kernels captured in the graph."""
_count = 0
_enabled = True


def add(n: int = 1):
    global _count
    if _enabled:
        _count += n


def get() -> int:
    return _count


def reset():
    global _count
    _count = 0


def count_graph(fn, *args, **kwargs):
    """Run fn once with counting on and return (result, launches it made):
    used to know how many kernels a captured graph replays."""
    before = get()
    out = fn(*args, **kwargs)
    return out, get() - before
