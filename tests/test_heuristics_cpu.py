"""Launch-shape heuristics of the attention kernels (pure host logic)."""
import importlib

ops = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops")


def test_prefill_tiles_cover_every_query_longest_first():
    q_lens = [1024, 300, 5]
    t = ops.prefill_tiles(q_lens).tolist()
    bq = ops.PREFILL_BQ
    # every (request, offset) tile once, offsets step by the tile height
    want = {(r, off) for r, n in enumerate(q_lens) for off in range(0, n, bq)}
    assert {tuple(x) for x in t} == want and len(t) == len(want)
    # causal: tiles with larger offsets see more keys and go first
    offs = [off for _, off in t]
    assert offs == sorted(offs, reverse=True)


def test_prefill_splits_only_when_sms_would_idle():
    # 32 heads x 4 tiles = 128 CTAs > 148/2: no split
    assert ops.prefill_splits(4, 32, 4096) == 1
    # 2 heads (TP=16-like) x 4 tiles: split to cover the SMs, >= 512 keys per split, <= 16
    s = ops.prefill_splits(4, 2, 8192)
    assert 1 < s <= 16 and 8192 // s >= 512
    assert ops.prefill_splits(4, 2, 600) == 1  # too few keys to split


def test_decode_splits_fill_sms_with_256_key_floor():
    assert ops.decode_splits(64, 8, 4096) == 1            # 512 (batch, head) pairs already fill 148 SMs
    s = ops.decode_splits(1, 1, 4096)
    assert s == min(2 * 148, 4096 // 256, 64) == 16       # bs=1 at TP=8: 16 splits of 256 keys
    assert ops.decode_splits(1, 1, 100) == 1              # short context: one split
    assert ops.decode_splits(1, 1, 1 << 20) == 64         # capped
