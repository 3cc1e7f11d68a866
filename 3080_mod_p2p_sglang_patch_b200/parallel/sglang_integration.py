"""Drop-in hook for sglang's ``dispatch_custom_allreduce``.

The reference wires itself into sglang with three lines at the top of
``dispatch_custom_allreduce()`` (sglang/README.md:14-31): when
``SGLANG_MAILBOX_AR`` is true it returns the ``MailboxAR`` class, which the
TP GroupCoordinator instantiates as ``ca_comm``. This module provides the same
function so a patched sglang can call it::

    from <this package>.parallel.sglang_integration import dispatch_custom_allreduce
    cls = dispatch_custom_allreduce()   # MailboxAR or None
"""
import logging

from ..config import mailbox_enabled
from .communicator import MailboxAR

logger = logging.getLogger(__name__)


def dispatch_custom_allreduce(default=None):
    """Return ``MailboxAR`` when ``SGLANG_MAILBOX_AR=1``, else ``default``."""
    if mailbox_enabled():
        logger.info("[AR] Using MailboxAR (NVLink symmetric-memory mode)")
        return MailboxAR
    return default
