"""Communicator configuration and environment flags.

Same switches as the reference (``SGLANG_MAILBOX_AR`` enables the communicator,
``SGLANG_MAILBOX_AR_VERBOSE`` turns on build/setup logging,
sglang/README.md:20 and sglang/mailbox_all_reduce.py:41) plus the knobs the
B200 design adds: buffer sizes, per-TP algorithm thresholds, the device wait
bound and an NVLS switch.
"""
import dataclasses
import os

MiB = 1 << 20

# Reference default for the largest message handled in-house (one 24 MB half,
# sglang/mailbox_all_reduce.py:20). Larger messages go through the chunked
# path up to ``max_size`` here.
REFERENCE_MAX_SIZE = 24 * MiB


def env_flag(name: str, default: bool = False) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")


def mailbox_enabled() -> bool:
    """``SGLANG_MAILBOX_AR=1`` turns the communicator on (reference flag)."""
    return env_flag("SGLANG_MAILBOX_AR", False)


@dataclasses.dataclass
class CommConfig:
    # largest message (bytes) handled by the communicator; above it the caller
    # falls back to NCCL. The kernels chunk through the buffer, so this is a
    # policy limit, not a buffer limit. None = per world size from
    # ``max_size_by_world``: the size where NCCL's pipelined ring overtakes the
    # in-house kernels on an 8xB200 NVSwitch box (benchmarks/allreduce_sweep.py,
    # graph mode: TP=2 32 MB 79 us vs NCCL 84, 64 MB 158 vs 152; TP=4 16 MB 56 vs
    # 72, 32 MB 121 vs 121, 64 MB 231 vs 188; TP=8 64 MB 259 vs 276, 128 MB 518
    # vs 395).
    max_size: int = None
    max_size_by_world: dict = dataclasses.field(
        default_factory=lambda: {2: 48 * MiB, 3: 32 * MiB, 4: 32 * MiB, 5: 96 * MiB, 6: 96 * MiB, 7: 96 * MiB,
                                 8: 96 * MiB}
    )
    # one ping-pong data half of the symmetric buffer (two halves are mapped)
    half_bytes: int = 64 * MiB
    # fused GEMM->allreduce path: one of its two halves (holds W partial slots
    # plus the reduced rows: 2 * M * N * 2 bytes for an [M, N] bf16 output)
    fuse_half_bytes: int = 40 * MiB
    # segmented (overlap) path: bytes per slot per source rank (0 disables)
    seg_slot_bytes: int = 8 * MiB
    # second communication lane (MailboxAR.lane): one ping-pong half of its
    # region, which has its own signal words and epochs (0 disables)
    lane_half_bytes: int = 32 * MiB
    # grid cap of a lane's allreduce + norm: leaves SMs to the other lane's compute
    lane_max_blocks: int = 64
    # bound of every device-side wait (the reference uses ~1 s, mailbox_ar_ext.cu:5)
    timeout_ns: int = 2_000_000_000
    # bound of host-side handshakes (FD exchange)
    handshake_timeout_ms: int = 60_000
    # use NVLS (multimem) when the GPUs expose multicast
    nvls: bool = True
    # one-shot (push) is used up to this many bytes, per world size
    oneshot_max: dict = dataclasses.field(
        default_factory=lambda: {2: 32 * MiB, 3: 2 * MiB, 4: 2 * MiB, 5: 1 * MiB, 6: 1 * MiB, 7: 1 * MiB, 8: 1 * MiB}
    )
    # NVLS is preferred over two-shot push at/above this many bytes on
    # ``nvls_min_world`` ranks or more (TP=8: 32 MB 130 us vs 142, 64 MB 260 vs
    # 268; TP=4: never faster, 64 MB 255 vs 231)
    nvls_min: int = 32 * MiB
    nvls_min_world: int = 8
    # grid cap of the allreduce kernels (blocks)
    max_blocks: int = 148
    # CPU transport: bytes per slot of the shared-memory mailbox
    cpu_slot_bytes: int = 32 * MiB
    cpu_timeout_ms: int = 30_000
    verbose: bool = False

    def max_size_for(self, world: int) -> int:
        if self.max_size is not None:
            return int(self.max_size)
        return int(self.max_size_by_world.get(world, 64 * MiB))

    @classmethod
    def from_env(cls) -> "CommConfig":
        c = cls()
        if "MBX_MAX_SIZE" in os.environ:
            c.max_size = int(os.environ["MBX_MAX_SIZE"])
        if "MBX_HALF_BYTES" in os.environ:
            c.half_bytes = int(os.environ["MBX_HALF_BYTES"])
        if "MBX_TIMEOUT_MS" in os.environ:
            c.timeout_ns = int(float(os.environ["MBX_TIMEOUT_MS"]) * 1e6)
        if "MBX_NVLS" in os.environ:
            c.nvls = env_flag("MBX_NVLS", True)
        if os.environ.get("NCCL_NVLS_ENABLE", "1") == "0":
            # a run that turned NVLS off for NCCL wants it off everywhere
            c.nvls = False
        if "MBX_MAX_BLOCKS" in os.environ:
            c.max_blocks = int(os.environ["MBX_MAX_BLOCKS"])
        if "MBX_LANE_MAX_BLOCKS" in os.environ:
            c.lane_max_blocks = int(os.environ["MBX_LANE_MAX_BLOCKS"])
        c.verbose = env_flag("SGLANG_MAILBOX_AR_VERBOSE", False)
        return c
