"""The class returned by ``dispatch_custom_allreduce`` driven the way sglang's
GroupCoordinator drives its ``ca_comm`` (the reference's integration,
sglang/README.md:14-31): constructed with keyword arguments on the TP CPU
group, asked ``should_custom_ar`` before each allreduce, ``custom_all_reduce``
returning None when it declines (the caller then uses its own collective),
``capture()`` around graph capture, ``register_graph_buffers()``, ``close()``.
Two gloo ranks on the CPU transport."""
import importlib
import os

import torch

from _mp import run_ranks

PKG = "3080_mod_p2p_sglang_patch_b200"


def _group_coordinator_flow(rank, world):
    import torch.distributed as dist

    os.environ["SGLANG_MAILBOX_AR"] = "1"
    integ = importlib.import_module(f"{PKG}.parallel.sglang_integration")
    cpu_group = dist.new_group(backend="gloo")
    ca_cls = integ.dispatch_custom_allreduce()
    ca = ca_cls(group=cpu_group, device=torch.device("cpu"), max_size=1 << 20)
    out = {"disabled": ca.disabled}

    def all_reduce(x):  # GroupCoordinator.all_reduce, reduced to its custom-AR branch
        if ca is not None and not ca.disabled and ca.should_custom_ar(x):
            y = ca.custom_all_reduce(x)
            if y is not None:
                return y, "custom"
        x = x.clone()
        dist.all_reduce(x, group=cpu_group)
        return x, "fallback"

    small = torch.full((4096,), float(rank + 1), dtype=torch.bfloat16)
    big = torch.full((1 << 20,), float(rank + 1), dtype=torch.float32)    # 4 MB > max_size
    odd = torch.ones(7, dtype=torch.bfloat16)                             # 14 bytes: not a multiple of 16
    for name, x in (("small", small), ("big", big), ("odd", odd)):
        y, path = all_reduce(x)
        out[name] = (path, float(y.float().mean()))
    out["declined_returns_none"] = ca.custom_all_reduce(big) is None
    with ca.capture():          # sglang enters this around CUDA-graph capture
        y, path = all_reduce(small)
    out["in_capture"] = path
    ca.register_graph_buffers()  # nothing to register: the buffers never move
    ca.close()
    out["closed"] = ca.disabled
    os.environ["SGLANG_MAILBOX_AR"] = "0"
    out["off"] = integ.dispatch_custom_allreduce("default")
    return out


def test_sglang_group_coordinator_flow_on_two_ranks():
    res = run_ranks(_group_coordinator_flow, 2)
    for r in (0, 1):
        o = res[r]
        assert o["disabled"] is False
        assert o["small"] == ("custom", 3.0)        # 1 + 2 on every element
        assert o["big"] == ("fallback", 3.0)        # above max_size: the caller's collective
        assert o["odd"] == ("fallback", 2.0)        # not 16-byte sized: declined
        assert o["declined_returns_none"] is True
        assert o["in_capture"] == "custom"
        assert o["closed"] is True and o["off"] == "default"


def test_dropin_module_exports_the_communicator():
    """The file a user copies into sglang's device_communicators/ exports this
    package's MailboxAR under the reference's module name."""
    import importlib.util

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        PKG, "integrations", "sglang", "mailbox_all_reduce.py")
    spec = importlib.util.spec_from_file_location("mailbox_all_reduce", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.MailboxAR is importlib.import_module(f"{PKG}.parallel").MailboxAR
