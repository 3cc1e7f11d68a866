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


@pytest.mark.parametrize("nq,nkv,splits", [(32, 8, 8), (8, 1, 16)])
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
        assert err < 2e-2, f"call {call}: max err {err}"


def test_noalloc_rejects_oversize_request():
    lib = _lib()
    cap = lib.mbx_decode_attention_noalloc_max_rows()
    q, kc, vc, kvl, bt = _inputs(1, [64] * 4, 32, 8)
    out = torch.empty_like(q)
    splits = cap // (4 * 32) + 1  # one row past the scratch
    rc = _call(lib, q, kc, vc, out, kvl, bt, splits)
    assert rc == 2
    assert b"exceeds the fixed scratch" in lib.mbx_noalloc_last_error()
