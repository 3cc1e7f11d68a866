"""Host side of the overlapped micro-batch prefill: how a ragged batch is cut
into two micro-batches (``LLMEngine._attn_halves``) and where the model splits
(``LlamaTP.overlap_split``). The kernels these feed run on the GPU; the
multi-GPU suite checks the overlapped forward against the plain one."""
import types

import torch

from conftest import sub


def _fake_engine(T1):
    eng_mod = sub("engine.engine")
    model = types.SimpleNamespace(overlap_split=lambda T: T1, scale=0.1)
    e = types.SimpleNamespace(model=model, cfg=types.SimpleNamespace(heads=32), tp_size=2,
                              device=torch.device("cpu"))
    e._h2d = lambda t: t
    return eng_mod.LLMEngine, e


def _meta(fn):
    d = fn.__defaults__
    cu, kvl, bt, tiles, splits = d
    return cu.tolist(), kvl.tolist(), bt, tiles, splits


def test_single_piece_split_in_half():
    cls, e = _fake_engine(512)
    bt = torch.arange(3 * 64, dtype=torch.int32).view(3, 64)[:1]
    T1, a0, a1 = cls._attn_halves(e, [1024], [3072], bt, 1024)
    assert T1 == 512
    cu0, kv0, bt0, _, _ = _meta(a0)
    cu1, kv1, bt1, _, _ = _meta(a1)
    # first half: rows 0..511 of the chunk, keys up to 3072 - 512; second: all keys
    assert cu0 == [0, 512] and kv0 == [2560]
    assert cu1 == [0, 512] and kv1 == [3072]
    assert torch.equal(bt0, bt) and torch.equal(bt1, bt)


def test_ragged_batch_cut_at_the_split():
    cls, e = _fake_engine(256)
    q_lens, kv_lens = [100, 300, 50], [100, 700, 1050]
    bt = torch.arange(3 * 8, dtype=torch.int32).view(3, 8)
    T1, a0, a1 = cls._attn_halves(e, q_lens, kv_lens, bt, sum(q_lens))
    cu0, kv0, bt0, _, _ = _meta(a0)
    cu1, kv1, bt1, _, _ = _meta(a1)
    # piece 0 whole (100 rows), piece 1's first 156 rows; then its last 144, piece 2
    assert cu0 == [0, 100, 256] and kv0 == [100, 700 - 144]
    assert cu1 == [0, 144, 194] and kv1 == [700, 1050]
    assert torch.equal(bt0, bt[[0, 1]]) and torch.equal(bt1, bt[[1, 2]])
    # every query row lands in exactly one micro-batch, in order
    assert cu0[-1] + cu1[-1] == sum(q_lens)


def test_no_split_when_the_model_declines():
    cls, e = _fake_engine(None)
    assert cls._attn_halves(e, [300], [300], torch.zeros(1, 4, dtype=torch.int32), 300) is None


def test_model_split_rows():
    models = sub("models")
    m = models.LlamaTP.__new__(models.LlamaTP)
    m.overlap_min_rows, m.sp, m.sp_min_rows = 512, None, 256
    m.cfg = types.SimpleNamespace(hidden=4096)
    limit = [64 << 20]
    lane = types.SimpleNamespace(fits_rmsnorm=lambda n: n <= limit[0])
    m.tp = types.SimpleNamespace(ca_comm=types.SimpleNamespace(fused_rmsnorm_limit=lambda: 1 << 30, lane=lambda: lane))
    assert m.overlap_split(1024) == 512
    assert m.overlap_split(700) == 256
    assert m.overlap_split(511) is None
    # each micro-batch's rows must fit the second lane's buffer
    limit[0] = 512 * 4096 * 2 - 1
    assert m.overlap_split(1024) is None
    m.overlap_min_rows = None
    assert m.overlap_split(4096) is None


def test_workspace_lanes_are_separate():
    """Kernels issued for the second micro-batch get their own split-K and
    split-KV scratch; the error word is shared."""
    ops = sub("ops")
    saved = dict(ops._WS)
    try:
        ops._WS.clear()
        made = []

        class FakeWs:
            def __init__(self, device, err=None):
                self.err = err if err is not None else object()
                made.append(self)

        orig = ops._Workspace
        ops._Workspace = FakeWs
        try:
            w0 = ops.workspace(0)
            with ops.workspace_lane(1):
                w1 = ops.workspace(0)
                assert ops.workspace(0) is w1
            assert ops.workspace(0) is w0
        finally:
            ops._Workspace = orig
        assert w0 is not w1 and w1.err is w0.err
    finally:
        ops._WS.clear()
        ops._WS.update(saved)
