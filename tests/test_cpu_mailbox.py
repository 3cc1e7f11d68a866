"""The mailbox lockstep protocol on CPU/gloo ranks.

Two (and four) processes run the communicator's CPU transport (native shared-
memory engine, csrc/cpu/mailbox_cpu.cpp) on fp32 and bf16 tensors of shape
[T, 4096], T in {1, 8, 256, 1024}, N(0,1) values seeded per rank, for 560
back-to-back rounds, each checked against torch.distributed.all_reduce.
Messages above the size limit must take the fallback path. The reference's
equivalents are tests/hammer_mbx.py (560 rounds) and tests/test_mailbox_torch.py.
"""
import pytest
import torch

from _mp import run_ranks

SHAPES_T = [1, 8, 256, 1024]


def _hammer(rank, world, rounds, dtype_name):
    import importlib

    import torch.distributed as dist

    mbx = importlib.import_module("3080_mod_p2p_sglang_patch_b200")
    from importlib import import_module

    comm_mod = import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    cfg = import_module("3080_mod_p2p_sglang_patch_b200.config").CommConfig()
    cfg.max_size = 4 * 1024 * 1024  # [256,4096] fp32 = 4 MiB fits, [1024,4096] fp32 = 16 MiB falls back
    ar = comm_mod.MailboxAR(None, "cpu", config=cfg)
    assert not ar.disabled, "CPU mailbox should come up"
    dtype = getattr(torch, dtype_name)
    g = torch.Generator().manual_seed(1000 * rank)
    n_custom = n_fallback = 0
    for it in range(rounds):
        T = SHAPES_T[it % len(SHAPES_T)]
        x = torch.randn(T, 4096, generator=g).to(dtype)
        ref = x.float().clone()
        dist.all_reduce(ref)
        if ar.should_custom_ar(x):
            out = ar.custom_all_reduce(x)
            n_custom += 1
        else:
            out = ar.all_reduce(x)
            n_fallback += 1
        tol = 1e-5 if dtype == torch.float32 else 2e-2
        assert torch.allclose(out.float(), ref, rtol=tol, atol=tol * 4), f"round {it} T={T} mismatch"
    epoch = ar.epoch()
    counters = dict(ar.counters)
    ar.close()
    return n_custom, n_fallback, epoch, counters, mbx.__version__


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_cpu_mailbox_560_rounds(world, dtype_name):
    rounds = 560 if world == 2 else 140
    res = run_ranks(_hammer, world, args=(rounds, dtype_name))
    n_custom, n_fallback, epoch, counters, _ = res[0]
    assert n_custom + n_fallback == rounds
    assert epoch == n_custom  # one protocol round per in-house call
    if dtype_name == "float32":
        assert n_fallback == rounds // 4  # every [1024,4096] fp32 message is over the limit
    assert counters["fallback"] == n_fallback
    assert all(r[:3] == res[0][:3] for r in res.values())


def _bitexact(rank, world):
    from importlib import import_module

    comm_mod = import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    ar = comm_mod.MailboxAR(None, "cpu")
    torch.manual_seed(1234)  # same values on every rank -> exact 2x (reference test_mailbox_torch.py:34-41)
    for it in range(100):
        nbytes = 4096 * (1 + (it * 37) % 300)
        x = torch.randn(nbytes // 2).to(torch.bfloat16)
        out = ar.custom_all_reduce(x)
        assert out is not None
        assert torch.equal(out, (x.float() * world).to(torch.bfloat16)), f"it {it}"
    ar.close()
    return True


def test_cpu_mailbox_bitexact_sum():
    run_ranks(_bitexact, 2)


def _gating(rank, world):
    from importlib import import_module

    comm_mod = import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    ar = comm_mod.MailboxAR(None, "cpu", max_size=1 << 16)
    ok = []
    ok.append(ar.should_custom_ar(torch.zeros(8, dtype=torch.float32)))           # 32 B: yes
    ok.append(ar.should_custom_ar(torch.zeros(3, dtype=torch.float32)))           # 12 B: not 16-aligned
    ok.append(ar.should_custom_ar(torch.zeros(8, dtype=torch.int32)))             # dtype
    ok.append(ar.should_custom_ar(torch.zeros(1 << 15, dtype=torch.float32)))     # 128 KiB > max_size
    ok.append(ar.should_custom_ar(torch.zeros(16, 16)[:, :8]))                    # not weak-contiguous
    ok.append(ar.custom_all_reduce(torch.zeros(3)) is None)                       # gated off -> None
    ar.close()
    return ok


def test_gating_matches_reference_rules():
    res = run_ranks(_gating, 2)
    assert res[0] == [True, False, False, False, False, True]


def _wrap(rank, world):
    import importlib

    comm_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    ar = comm_mod.MailboxAR(None, "cpu")
    ar.debug_set_epoch((1 << 32) - 20)
    bad = 0
    for it in range(60):
        v = float(it % 251 + 1)
        out = ar.custom_all_reduce(torch.full((8192,), v * (rank + 1)))
        bad += int(not bool(torch.all(out == v * sum(range(1, world + 1)))))
    ep = ar.epoch()
    ar.close()
    return bad, ep


def test_epoch_wraps_past_2_pow_32():
    """60 rounds starting 20 below 2^32: the wrap-safe epoch compare keeps
    every wait correct across the wrap (a plain >= would pass stale flags)."""
    res = run_ranks(_wrap, 2)
    for r in (0, 1):
        assert res[r] == (0, 40), res
