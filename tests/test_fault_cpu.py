"""Failure detection without a GPU fault: a rank skips a round, the peer's
bounded wait gives up and raises MailboxError; a collective reset() brings the
group back. The reference's equivalent is the device timeout -> err code path
(sglang/mailbox_ar_ext.cu:25-45), which it never checks on the host."""
import torch

from _mp import run_ranks


def _skip_round(rank, world):
    from importlib import import_module

    comm_mod = import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    cfg = import_module("3080_mod_p2p_sglang_patch_b200.config").CommConfig()
    cfg.cpu_timeout_ms = 300
    ar = comm_mod.MailboxAR(None, "cpu", config=cfg)
    x = torch.ones(1024)
    for _ in range(5):
        assert torch.equal(ar.custom_all_reduce(x), x * world)
    raised = False
    if rank == 0:  # rank 1 "drops" this round
        try:
            ar.custom_all_reduce(x)
        except comm_mod.MailboxError:
            raised = True
    err = ar.err()
    ar.reset()
    for _ in range(5):
        assert torch.equal(ar.custom_all_reduce(x), x * world)
    healthy = ar.check_health()
    ar.close()
    return raised, err, healthy


def test_skipped_round_times_out_and_recovers():
    res = run_ranks(_skip_round, 2)
    assert res[0][0] is True and res[0][1] == 3
    assert res[1][0] is False
    assert res[0][2] and res[1][2]


def _bad_world(rank, world):
    from importlib import import_module

    comm_mod = import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    import torch.distributed as dist

    sub = dist.new_group([0])  # a 1-rank group: nothing to reduce -> disabled, caller uses NCCL
    ar = comm_mod.MailboxAR(sub, "cpu") if rank == 0 else None
    return ar.disabled if ar is not None else True


def test_world_size_one_is_disabled():
    res = run_ranks(_bad_world, 2)
    assert res[0] is True


def _inject(rank, world, spec):
    import os
    from importlib import import_module

    os.environ["MBX_INJECT_FAULT"] = spec
    comm_mod = import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    ar = comm_mod.MailboxAR(None, "cpu")
    os.environ.pop("MBX_INJECT_FAULT")
    x = torch.full((4096,), float(rank + 1))
    out = ar.all_reduce(x)  # in-house when up, gloo fallback otherwise
    res = (ar.disabled, getattr(ar, "_attempt", None), bool(torch.all(out == sum(range(1, world + 1)))))
    ar.close()
    return res


def test_one_rank_open_failure_retries_on_every_rank():
    """Rank 1 fails to map the mailbox at attempt 0 only: every rank retries
    and comes up at attempt 1 (the consensus makes rank 0 drop its good
    mapping too)."""
    res = run_ranks(_inject, 2, args=("cpu_open@1#0",))
    for r in (0, 1):
        assert res[r] == (False, 1, True), res


def test_persistent_failure_falls_back_to_nccl_on_every_rank():
    """Rank 2 of 3 can never map the mailbox: all three ranks disable the
    communicator (no hang, no split decision) and the allreduce still works
    through the process-group fallback."""
    res = run_ranks(_inject, 3, args=("cpu_open@2",))
    for r in (0, 1, 2):
        assert res[r][0] is True and res[r][2] is True, res
