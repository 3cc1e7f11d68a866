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
