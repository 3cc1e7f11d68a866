"""Parallel runtime: symmetric memory, the MailboxAR communicator, TP groups."""
from .communicator import (ALGO_NAMES, ALGO_NVLS, ALGO_ONESHOT_PULL, ALGO_ONESHOT_PUSH, ALGO_TWOSHOT,  # noqa: F401
                           ALGO_TWOSHOT_PUSH, DTYPE_IDS,
                           MailboxAR, MailboxError, is_weak_contiguous)
from .sglang_integration import dispatch_custom_allreduce  # noqa: F401
from .tp import TPGroup, init_distributed  # noqa: F401
