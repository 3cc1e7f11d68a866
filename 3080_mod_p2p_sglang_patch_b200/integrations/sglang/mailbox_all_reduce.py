"""Drop-in ``mailbox_all_reduce.py`` for sglang: the ``MailboxAR`` that
sglang's TP group coordinator instantiates as ``ca_comm``, backed by this
package's NVLink communicator (the same module name and class name as the
reference's sglang/mailbox_all_reduce.py, so its wiring is unchanged).

Install (this package importable, e.g. ``pip install -e <repo>`` or on
PYTHONPATH)::

    SGC=$(python3 -c 'import sglang,os;print(os.path.dirname(sglang.__file__))')
    cp mailbox_all_reduce.py $SGC/srt/distributed/device_communicators/

then, at the top of ``dispatch_custom_allreduce()`` in
``custom_all_reduce.py`` of that directory::

    if _is_cuda and get_bool_env_var("SGLANG_MAILBOX_AR", default="false"):
        from .mailbox_all_reduce import MailboxAR
        logger.info("[AR] Using MailboxAR (NVLink symmetric-memory mode)")
        return MailboxAR

and launch with ``SGLANG_MAILBOX_AR=1 python -m sglang.launch_server ... --tp N``.
No CUDA extension is compiled at startup: the kernels ship prebuilt with the
package.
"""
from mailbox_ar_b200.parallel import MailboxAR, is_weak_contiguous  # noqa: F401

__all__ = ["MailboxAR", "is_weak_contiguous"]
