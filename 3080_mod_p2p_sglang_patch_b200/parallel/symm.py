"""Symmetric buffers: one fixed-address buffer per rank, mapped by every rank.

Replaces the reference's driver-patched BAR1 mailbox and its 16-attempt
"window landing" loop (driver/p2p-mailbox-595.91.07.patch:797-970,
sglang/mailbox_all_reduce.py:91-146). On B200 every peer is reachable over
NVLink 5 / NVSwitch, so each rank:

1. allocates its buffer with cuMemCreate (POSIX-FD shareable) and zeroes it,
2. sends the FD to every peer and imports theirs (mapped once, fixed VA),
3. optionally binds all buffers to one NVLS multicast object (multimem access).

If the VMM path fails on any rank, every rank retries with the legacy CUDA IPC
handle path (cudaIpcGetMemHandle / cudaIpcOpenMemHandle, the reference's
transport) so the group stays consistent.
"""
import logging
import os

import torch
import torch.distributed as dist

from .._ext import cuda_ext
from . import bootstrap, faults

logger = logging.getLogger(__name__)


def _round_up(x, g):
    return (x + g - 1) // g * g


class SymmetricBuffer:
    """Fixed-address symmetric buffer over a process group.

    Attributes: ``ptrs`` (every rank's buffer base in this process),
    ``local_ptr``, ``mc_ptr`` (NVLS mapping or 0), ``size``, ``transport``
    ("vmm" or "ipc").
    """

    def __init__(self, size: int, device: torch.device, group=None, nvls: bool = True, timeout_ms: int = 60000,
                 session: str = None):
        self.C = cuda_ext()
        self.group = group
        self.rank = dist.get_rank(group=group)
        self.world = dist.get_world_size(group=group)
        self.device = device
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.mc_ptr = 0
        self._mc_id = 0
        self._mc_joined = False  # every rank's device was added to the multicast object
        self._mc_bound = False  # this rank's buffer is bound to the multicast object
        self._ids = []
        self._ipc_ptrs = []
        self._ipc_tensor = None
        self.transport = None
        session = session or bootstrap.session_id(group)
        want_mc = bool(nvls) and self.world > 1
        mc_ok_local = False
        if want_mc:
            try:
                mc_ok_local = bool(self.C.mc_supported(self.dev))
            except Exception:  # noqa: BLE001
                mc_ok_local = False
        use_mc = bootstrap.agree(mc_ok_local, group) if want_mc else False
        gran = 2 << 20
        err = None
        try:
            gran = int(self.C.symm_granularity(self.dev, use_mc, self.world))
        except Exception as e:  # noqa: BLE001
            err = e
        grans = bootstrap.all_gather_obj(gran, group)
        self.size = _round_up(size, max(grans))
        if bootstrap.agree(err is None, group):
            try:
                self._setup_vmm(session, timeout_ms)
                self.transport = "vmm"
            except Exception as e:  # noqa: BLE001
                logger.warning("[MailboxAR] VMM symmetric buffer failed (%s); trying CUDA IPC", e)
                self._free_vmm()
        if self.transport is None:
            self._setup_ipc()
            self.transport = "ipc"
            use_mc = False
        if use_mc:
            try:
                self._setup_nvls(session, timeout_ms)
            except Exception as e:  # noqa: BLE001
                logger.warning("[MailboxAR] NVLS multicast setup failed (%s); continuing without it", e)
                self._release_mc()

    # ------------------------------------------------------------------ VMM
    def _setup_vmm(self, session, timeout_ms):
        C = self.C
        err = None
        mine = None
        try:
            faults.check("symm_create", self.rank)
            mine = C.symm_create(self.dev, self.size)
            self._ids.append(mine.id)
        except Exception as e:  # noqa: BLE001
            err = e
        if not bootstrap.agree(err is None, self.group):
            if mine is not None and mine.fd >= 0:
                C.close_fd(mine.fd)
            raise RuntimeError(f"cuMemCreate failed on some rank ({err})")
        try:
            fds = bootstrap.exchange_fds(session, self.rank, self.world, mine.fd, self.group, timeout_ms, "mem")
        finally:
            C.close_fd(mine.fd)
        ptrs = [0] * self.world
        ptrs[self.rank] = mine.ptr
        self._mem_id = mine.id
        err = None
        try:
            faults.check("symm_import", self.rank)
            for p, fd in sorted(fds.items()):
                try:
                    a = C.symm_import(self.dev, fd, self.size)
                finally:
                    os.close(fd)
                self._ids.append(a.id)
                ptrs[p] = a.ptr
        except Exception as e:  # noqa: BLE001
            err = e
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"importing peer buffers failed on some rank ({err})")
        self.ptrs = ptrs
        self.local_ptr = ptrs[self.rank]

    def _free_vmm(self):
        for i in reversed(self._ids):
            try:
                self.C.symm_free(i)
            except Exception:  # noqa: BLE001
                pass
        self._ids = []

    # ------------------------------------------------------------------ NVLS
    def _setup_nvls(self, session, timeout_ms):
        C = self.C
        err = None
        fd = -1
        if self.rank == 0:
            try:
                mc = C.mc_create(self.world, self.size)
                self._mc_id = mc.id
                fd = mc.fd
            except Exception as e:  # noqa: BLE001
                err = e
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"cuMulticastCreate failed ({err})")
        rfd = bootstrap.broadcast_fd(session, self.rank, self.world, fd, 0, self.group, timeout_ms, "mc")
        try:
            if self.rank != 0:
                faults.check("mc_import", self.rank)
                self._mc_id = C.mc_import(rfd, self.size)
            C.mc_add_device(self._mc_id, self.dev)
        except Exception as e:  # noqa: BLE001
            err = e
        finally:
            if rfd >= 0:
                C.close_fd(rfd)
        # every device must be added before any memory is bound
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"cuMulticastAddDevice failed ({err})")
        self._mc_joined = True
        try:
            C.mc_bind(self._mc_id, self._mem_id, self.size)
            self._mc_bound = True
        except Exception as e:  # noqa: BLE001
            err = e
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"cuMulticastBindMem failed ({err})")
        try:
            self.mc_ptr = C.mc_map(self._mc_id, self.dev, self.size)
        except Exception as e:  # noqa: BLE001
            err = e
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"mapping the multicast object failed ({err})")

    # ------------------------------------------------------------------ IPC
    def _setup_ipc(self):
        C = self.C
        self._ipc_tensor = torch.zeros(self.size, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)
        h = C.ipc_get_handle(self._ipc_tensor.data_ptr())
        handles = bootstrap.all_gather_obj(h, self.group)
        ptrs = [0] * self.world
        ptrs[self.rank] = self._ipc_tensor.data_ptr()
        err = None
        try:
            faults.check("ipc_open", self.rank)
            for p in range(self.world):
                if p != self.rank:
                    ptrs[p] = C.ipc_open(handles[p])
                    self._ipc_ptrs.append(ptrs[p])
        except Exception as e:  # noqa: BLE001
            err = e
        if not bootstrap.agree(err is None, self.group):
            raise RuntimeError(f"CUDA IPC open failed on some rank ({err})")
        self.ptrs = ptrs
        self.local_ptr = ptrs[self.rank]

    def zero_signals(self, nbytes: int):
        """Zero the first ``nbytes`` of the local buffer (signal area)."""
        torch.cuda.synchronize(self.device)
        _raw_uint8(self.local_ptr, nbytes, self.device).zero_()
        torch.cuda.synchronize(self.device)

    def _release_mc(self):
        """Drop this rank's multicast mapping, binding and handle, whatever
        stage the setup reached (unbinding is only valid after a bind)."""
        C = self.C
        if self._mc_bound:
            try:
                C.mc_unbind(self._mc_id, self.dev, self.size)
            except Exception:  # noqa: BLE001
                pass
            self._mc_bound = False
        if self._mc_id and self._mc_joined:
            try:
                C.symm_free(self._mc_id)  # unmaps the multicast range if mapped, releases the handle
            except Exception:  # noqa: BLE001
                pass
        # an object whose device set never completed is left to process exit
        # (no driver call on a half-built multicast object)
        self._mc_id = 0
        self._mc_joined = False
        self.mc_ptr = 0

    def close(self):
        C = self.C
        self._release_mc()
        self._free_vmm()
        for p in self._ipc_ptrs:
            try:
                C.ipc_close(p)
            except Exception:  # noqa: BLE001
                pass
        self._ipc_ptrs = []
        self._ipc_tensor = None


def _raw_uint8(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """A uint8 tensor view of raw device memory (no ownership)."""
    class _Holder:
        pass

    h = _Holder()
    h.__cuda_array_interface__ = {
        "shape": (nbytes,),
        "typestr": "|u1",
        "data": (ptr, False),
        "version": 3,
        "strides": None,
    }
    return torch.as_tensor(h, device=device)
