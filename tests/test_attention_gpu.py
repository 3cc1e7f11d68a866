"""Paged prefill (chunked, causal) and split-KV decode attention vs fp32."""

import pytest
import torch

from conftest import sub

pytestmark = pytest.mark.gpu

PAGE, D = 16, 128


def _paged(lengths, nkv, blocks_per_req, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    R = len(lengths)
    nblocks = R * blocks_per_req
    kc = torch.randn(nblocks, nkv, PAGE, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(nblocks, nkv, PAGE, D, device="cuda", generator=g).to(torch.bfloat16)
    perm = torch.randperm(nblocks, device="cuda", generator=g).to(torch.int32)
    bt = perm.view(R, blocks_per_req).contiguous()
    return kc, vc, bt


@pytest.mark.parametrize("kernel", ["tc", "tc_split4", "mma"])
@pytest.mark.parametrize("nq,nkv", [(32, 8), (4, 1), (8, 1)])
def test_prefill_chunked_ragged(nq, nkv, kernel):
    ops, ref = sub("ops"), sub("ops.reference")
    kv_lens = [100, 264, 1024, 777]
    q_lens = [100, 64, 300, 257]     # req 0 fresh, req 1/2/3 are later chunks (unaligned offsets)
    kc, vc, bt = _paged(kv_lens, nkv, 64)
    T = sum(q_lens)
    q = torch.randn(T, nq, D, device="cuda").to(torch.bfloat16)
    cu = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32, device="cuda")
    kvl = torch.tensor(kv_lens, dtype=torch.int32, device="cuda")
    if kernel.startswith("tc"):
        sp = 4 if kernel == "tc_split4" else 1
        out = ops.prefill_attention(q, kc, vc, cu, kvl, bt, ops.prefill_tiles(q_lens).cuda(), splits=sp)
    else:
        out = ops.prefill_attention_mma(q, kc, vc, cu, kvl, bt, ops.prefill_tiles(q_lens, bq=64).cuda())
    torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    for r in range(len(q_lens)):
        qs = q[cu[r]:cu[r + 1]]
        k = ref.gather_kv(kc, bt[r], kv_lens[r])
        v = ref.gather_kv(vc, bt[r], kv_lens[r])
        want = ref.attention(qs, k, v, causal_offset=kv_lens[r] - q_lens[r])
        err = (out[cu[r]:cu[r + 1]].float() - want).abs().max().item()
        assert err < 2e-2, f"request {r}: max err {err}"


@pytest.mark.parametrize("splits", [1, 4, 16])
@pytest.mark.parametrize("nq,nkv", [(32, 8), (4, 1), (8, 1)])
def test_decode_split_kv(splits, nq, nkv):
    ops, ref = sub("ops"), sub("ops.reference")
    lens = [1, 17, 500, 4096]
    kc, vc, bt = _paged(lens, nkv, 256, seed=1)
    B = len(lens)
    q = torch.randn(B, nq, D, device="cuda").to(torch.bfloat16)
    kvl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = ops.decode_attention(q, kc, vc, kvl, bt, splits=splits)
    torch.cuda.synchronize()
    for b in range(B):
        k = ref.gather_kv(kc, bt[b], lens[b])
        v = ref.gather_kv(vc, bt[b], lens[b])
        want = ref.attention(q[b:b + 1], k, v)
        err = (out[b:b + 1].float() - want).abs().max().item()
        assert err < 2e-2, f"b={b}: max err {err}"


@pytest.mark.parametrize("splits", [2, 7, 16])
def test_decode_in_kernel_merge_matches_combine_launch(splits):
    """The split-KV merge done by each (request, kv head)'s last CTA gives the
    bit-identical output of the separate combine launch, call after call (the
    arrival counts reset themselves)."""
    ops = sub("ops")
    C = sub("_ext").cuda_ext()
    lens = [3, 260, 4096, 1000, 17]
    nq, nkv = 32, 8
    kc, vc, bt = _paged(lens, nkv, 256, seed=5)
    B = len(lens)
    kvl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(B * nkv, dtype=torch.int32, device="cuda")
    po = torch.empty(B * nq * splits * D, device="cuda")
    pl = torch.empty(B * nq * splits, device="cuda")
    scale = 1.0 / D ** 0.5
    for it in range(3):
        q = torch.randn(B, nq, D, device="cuda").to(torch.bfloat16)
        want = torch.empty_like(q)
        C.decode_attention(q, kc, vc, want, kvl, bt, po, pl, splits, scale)
        got = torch.empty_like(q)
        C.decode_attention(q, kc, vc, got, kvl, bt, po, pl, splits, scale, cnt)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"iteration {it}"
        assert int(cnt.abs().sum().item()) == 0
    assert torch.equal(ops.decode_attention(q, kc, vc, kvl, bt, splits=splits), want)
