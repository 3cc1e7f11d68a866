"""Flags and configuration: the reference's SGLANG_MAILBOX_AR switch and
sglang hook (sglang/README.md:14-31), env overrides, the per-world NCCL
fallback size, and the fault-injection rule parser."""
import importlib

cfg_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.config")
integ = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel.sglang_integration")
faults = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel.faults")


def test_sglang_flag_selects_the_communicator(monkeypatch):
    monkeypatch.delenv("SGLANG_MAILBOX_AR", raising=False)
    assert integ.dispatch_custom_allreduce("nccl-default") == "nccl-default"
    for v in ("1", "true", "on"):
        monkeypatch.setenv("SGLANG_MAILBOX_AR", v)
        assert integ.dispatch_custom_allreduce() is integ.MailboxAR
    monkeypatch.setenv("SGLANG_MAILBOX_AR", "0")
    assert integ.dispatch_custom_allreduce() is None


def test_env_overrides(monkeypatch):
    monkeypatch.setenv("MBX_MAX_SIZE", str(8 << 20))
    monkeypatch.setenv("MBX_TIMEOUT_MS", "250")
    monkeypatch.setenv("MBX_NVLS", "0")
    monkeypatch.setenv("SGLANG_MAILBOX_AR_VERBOSE", "1")
    c = cfg_mod.CommConfig.from_env()
    assert c.max_size_for(8) == 8 << 20 and c.timeout_ns == 250_000_000 and c.nvls is False and c.verbose
    monkeypatch.delenv("MBX_NVLS")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")  # NVLS off for NCCL means off here too
    assert cfg_mod.CommConfig.from_env().nvls is False


def test_per_world_fallback_size(monkeypatch):
    for k in ("MBX_MAX_SIZE", "NCCL_NVLS_ENABLE"):
        monkeypatch.delenv(k, raising=False)
    c = cfg_mod.CommConfig.from_env()
    MiB = 1 << 20
    assert c.max_size_for(2) == 48 * MiB and c.max_size_for(4) == 32 * MiB and c.max_size_for(8) == 96 * MiB
    # the reference's own limit is smaller: everything it handled in-house stays in-house here
    assert all(c.max_size_for(w) >= cfg_mod.REFERENCE_MAX_SIZE for w in range(2, 9))


def test_fault_rules(monkeypatch):
    monkeypatch.setenv("MBX_INJECT_FAULT", "cpu_open@1#0, symm_import@0")
    faults.set_attempt(0)
    faults.check("cpu_open", 0)  # other rank: no fault
    try:
        faults.check("cpu_open", 1)
        raise AssertionError("expected an injected fault")
    except faults.InjectedFault:
        pass
    faults.set_attempt(1)
    faults.check("cpu_open", 1)  # only attempt 0
    try:
        faults.check("symm_import", 0)  # every attempt
        raise AssertionError("expected an injected fault")
    except faults.InjectedFault:
        pass
    monkeypatch.delenv("MBX_INJECT_FAULT")
    faults.check("symm_import", 0)
    faults.set_attempt(0)


def test_importable_alias_resolves_to_the_same_modules():
    """``mailbox_ar_b200.X`` is the package under an importable name: the
    same module objects (one copy of the extensions and their state)."""
    import mailbox_ar_b200.engine as e
    from mailbox_ar_b200.parallel import MailboxAR

    real = importlib.import_module("3080_mod_p2p_sglang_patch_b200")
    assert e is importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine")
    assert MailboxAR is integ.MailboxAR
    import mailbox_ar_b200
    assert mailbox_ar_b200.engine is real.engine


def test_algorithm_choice_by_size_and_world():
    """The measured routing: one-shot push up to oneshot_max, NVLS from
    nvls_min only on nvls_min_world ranks or more (and only with multicast),
    two-shot push otherwise."""
    import types

    comm = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    MiB = 1 << 20
    cfg = cfg_mod.CommConfig()

    def pick(world, nbytes, mc=True):
        ar = object.__new__(comm.MailboxAR)
        ar.cfg, ar.world_size = cfg, world
        ar._buf = types.SimpleNamespace(mc_ptr=1 if mc else 0)
        return comm.ALGO_NAMES[ar.pick_algo(nbytes)]

    assert pick(2, 32 * MiB) == "oneshot_push" and pick(2, 40 * MiB) == "twoshot_push"
    assert pick(4, 2 * MiB) == "oneshot_push" and pick(4, 4 * MiB) == "twoshot_push"
    assert pick(4, 64 * MiB) == "twoshot_push"  # NVLS never beat two-shot push at four ranks
    assert pick(8, 1 * MiB) == "oneshot_push" and pick(8, 16 * MiB) == "twoshot_push"
    assert pick(8, 32 * MiB) == "nvls" and pick(8, 32 * MiB, mc=False) == "twoshot_push"
