"""The allocation-free decode-attention entry point, called through its
exported C symbol (as a caller without PyTorch's allocator would), against the
regular entry point on the same inputs, twice in a row (the shared scratch
keeps the previous call's contents, which must not leak into the next call).

Collected last on purpose: if it fails, a run that stops at the first failure
has already run every other test."""
import ctypes
import glob
import os

import pytest
import torch

from conftest import ROOT, sub

pytestmark = pytest.mark.gpu

PAGE, D = 16, 128


def _lib():
    paths = glob.glob(os.path.join(ROOT, "3080_mod_p2p_sglang_patch_b200", "_C*.so"))
    assert paths, "the CUDA extension is not built"
    lib = ctypes.CDLL(paths[0])
    f = lib.mbx_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    lib.mbx_noalloc_last_error.restype = ctypes.c_char_p
    lib.mbx_decode_attention_noalloc_max_rows.restype = ctypes.c_size_t
    return lib


def _inputs(seed, lens, nq, nkv):
    g = torch.Generator(device="cuda").manual_seed(seed)
    B = len(lens)
    blocks_per = max(1, max(lens) // PAGE + 1)
    nblocks = B * blocks_per
    kc = torch.randn(nblocks, nkv, PAGE, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(nblocks, nkv, PAGE, D, device="cuda", generator=g).to(torch.bfloat16)
    bt = torch.randperm(nblocks, device="cuda", generator=g).to(torch.int32).view(B, blocks_per).contiguous()
    q = torch.randn(B, nq, D, device="cuda", generator=g).to(torch.bfloat16)
    kvl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, kvl, bt


def _call(lib, q, kc, vc, out, kvl, bt, splits):
    B, nq, _ = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return lib.mbx_decode_attention_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                            kvl.data_ptr(), bt.data_ptr(), bt.shape[1], B, nq, kc.shape[1],
                                            splits, 1.0 / D ** 0.5, stream)


def _fp32_reference(q, kc, vc, kvl, bt):
    """Plain fp32 attention of every batch row over its gathered pages."""
    ref = sub("ops.reference")
    rows = []
    for b, n in enumerate(kvl.tolist()):
        k = ref.gather_kv(kc, bt[b], n)
        v = ref.gather_kv(vc, bt[b], n)
        rows.append(ref.attention(q[b:b + 1], k, v))
    return torch.cat(rows, 0)


@pytest.mark.parametrize("nq,nkv,splits", [(32, 8, 8), (8, 1, 16), (32, 8, 1)])
def test_noalloc_matches_regular_entry_point_twice(nq, nkv, splits):
    ops = sub("ops")
    lib = _lib()
    for call, seed in enumerate((11, 12)):  # two calls in a row, different data
        lens = [1, 33, 700, 2048 + call * 100]
        q, kc, vc, kvl, bt = _inputs(seed, lens, nq, nkv)
        out = torch.full_like(q, float("nan"))
        rc = _call(lib, q, kc, vc, out, kvl, bt, splits)
        assert rc == 0, lib.mbx_noalloc_last_error().decode()
        want = ops.decode_attention(q, kc, vc, kvl, bt, splits=splits)
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        err = (out.float() - want.float()).abs().max().item()
        assert err < 2e-2, f"call {call}: max err {err} against the regular entry point"
        err32 = (out.float() - _fp32_reference(q, kc, vc, kvl, bt)).abs().max().item()
        assert err32 < 2e-2, f"call {call}: max err {err32} against fp32 attention"


def test_noalloc_single_split_has_no_row_limit():
    """One split writes the output directly: a batch whose rows exceed the
    scratch is still served (the limit only applies to split partials)."""
    ops = sub("ops")
    lib = _lib()
    cap = lib.mbx_decode_attention_noalloc_max_rows()
    nq, nkv = 32, 8
    B = cap // nq + 8
    q, kc, vc, kvl, bt = _inputs(5, [40] * B, nq, nkv)
    out = torch.full_like(q, float("nan"))
    rc = _call(lib, q, kc, vc, out, kvl, bt, 1)
    assert rc == 0, lib.mbx_noalloc_last_error().decode()
    want = ops.decode_attention(q, kc, vc, kvl, bt, splits=1)
    torch.cuda.synchronize()
    assert (out.float() - want.float()).abs().max().item() < 2e-2
    pick = [0, B // 2, B - 1]
    got = out[pick].float()
    ref = _fp32_reference(q[pick], kc, vc, kvl[pick], bt[pick])
    assert (got - ref).abs().max().item() < 2e-2


def test_noalloc_rejects_bad_group_and_null_pointers():
    lib = _lib()
    q, kc, vc, kvl, bt = _inputs(2, [64, 64], 12, 8)  # 12 query heads over 8 kv heads
    out = torch.empty_like(q)
    rc = _call(lib, q, kc, vc, out, kvl, bt, 4)
    assert rc == 4
    assert b"group size" in lib.mbx_noalloc_last_error()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mbx_decode_attention_noalloc(None, kc.data_ptr(), vc.data_ptr(), out.data_ptr(), kvl.data_ptr(),
                                          bt.data_ptr(), bt.shape[1], 2, 12, 8, 4, 0.1, stream)
    assert rc == 1
    assert b"null pointer" in lib.mbx_noalloc_last_error()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_second_device_after_first():
    """The scratch address and the kernel's shared-memory limit are per
    device: a call on device 1 after device 0 must work as well."""
    ops = sub("ops")
    lib = _lib()
    for dev in (0, 1):
        with torch.cuda.device(dev):
            q, kc, vc, kvl, bt = _inputs(20 + dev, [5, 300, 1500], 32, 8)
            out = torch.full_like(q, float("nan"))
            rc = _call(lib, q, kc, vc, out, kvl, bt, 8)
            assert rc == 0, lib.mbx_noalloc_last_error().decode()
            want = ops.decode_attention(q, kc, vc, kvl, bt, splits=8)
            torch.cuda.synchronize()
            assert (out.float() - want.float()).abs().max().item() < 2e-2


def test_noalloc_rejects_oversize_request():
    lib = _lib()
    cap = lib.mbx_decode_attention_noalloc_max_rows()
    q, kc, vc, kvl, bt = _inputs(1, [64] * 4, 32, 8)
    out = torch.empty_like(q)
    splits = cap // (4 * 32) + 1  # one row past the scratch
    rc = _call(lib, q, kc, vc, out, kvl, bt, splits)
    assert rc == 2
    assert b"exceeds the fixed scratch" in lib.mbx_noalloc_last_error()
