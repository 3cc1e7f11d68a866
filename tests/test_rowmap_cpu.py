"""Index arithmetic of the allreduce+RMSNorm row kernels (csrc/ar/allreduce.cu:
block_rows, for_norm_rows, for_owner_norm_rows and the phases of
ar_rmsnorm_twoshot_push / fused_rs_norm_kernel / ar_rmsnorm_oneshot_kernel),
restated in Python. The kernels synchronise phases with block-pairwise
barriers (block b of every rank waits only for block b of the others), which
is enough only if every row a phase reads was written by the same block
index in the previous phase, on every rank. This checks that invariant, and
that each phase covers every row exactly once, for 2-8 ranks and many row
counts (the 4- and 8-rank scaling runs use the same code as the 2-rank
GPU tests, with a different W)."""
import pytest

ROW_WARPS = 16      # kArThreads / 32
MAX_BLOCKS = 148    # default grid cap (CommConfig.max_blocks)


def block_rows(n, b, g):
    return (n - 1 - b) // g + 1 if n > b else 0


def norm_rows(count):
    """k values a block visits in for_norm_rows (whole block for one row, else one warp per row)."""
    if count == 1:
        return [0]
    return [k for w in range(ROW_WARPS) for k in range(w, count, ROW_WARPS)]


def owner_norm_rows(M, Mo, W, b, g):
    per = block_rows(Mo, b, g)
    rows = []
    for k in norm_rows(W * per):
        o, j = k // per, k % per
        row = o * Mo + b + j * g
        if row < min(M, o * Mo + Mo):
            rows.append(row)
    return rows


@pytest.mark.parametrize("W", [2, 3, 4, 5, 6, 7, 8])
def test_phases_read_only_rows_their_block_wrote(W):
    for M in (1, 2, 7, 9, 16, 17, 63, 64, 65, 128, 129, 255, 256, 333, 1000, 1024, 2048, 8192):
        Mo = (M + W - 1) // W
        g = max(1, min(Mo, MAX_BLOCKS))  # grid of the two-shot / fused launches
        writer = {}  # phase B (owned rows, reduced and pushed): row -> writing block
        for o in range(W):
            r0, r1 = o * Mo, min(M, o * Mo + Mo)
            for b in range(g):
                for j in range(block_rows(r1 - r0, b, g)):
                    row = r0 + b + j * g
                    assert row not in writer
                    writer[row] = b
        assert sorted(writer) == list(range(M))
        seen = []  # phase C (normalise every row): each read row was written by the same block index
        for b in range(g):
            for row in owner_norm_rows(M, Mo, W, b, g):
                assert writer[row] == b, (W, M, row, b)
                seen.append(row)
        assert sorted(seen) == list(range(M))
        # phase A (push rows to their owner) uses the same row -> block map as phase B
        for o in range(W):
            a0, a1 = o * Mo, min(M, o * Mo + Mo)
            for b in range(g):
                pushed = {a0 + b + j * g for j in range(block_rows(a1 - a0, b, g))}
                assert pushed == {r for r, bb in writer.items() if bb == b and a0 <= r < a1}
        # one-shot: grid from M; rows b + j*g pushed and later normalised by block b
        g1 = max(1, min(M, MAX_BLOCKS))
        cover = [b + k * g1 for b in range(g1) for k in norm_rows(block_rows(M, b, g1))
                 if block_rows(M, b, g1) > 0]
        assert sorted(cover) == list(range(M))
