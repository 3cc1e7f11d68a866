"""Elementwise sm_100a kernels vs PyTorch fp32 references."""
import pytest
import torch

from conftest import sub

pytestmark = pytest.mark.gpu


def test_rmsnorm_and_fused_add():
    ops, ref = sub("ops"), sub("ops.reference")
    torch.manual_seed(0)
    for M, H in [(1, 4096), (37, 4096), (1024, 8192)]:
        x = torch.randn(M, H, device="cuda").to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(H, device="cuda")).to(torch.bfloat16)
        out = ops.rmsnorm(x, w, 1e-5)
        assert (out.float() - ref.rmsnorm(x, w, 1e-5)).abs().max().item() < 3e-2
        r = torch.randn(M, H, device="cuda").to(torch.bfloat16)
        r0 = r.clone()
        out2 = ops.fused_add_rmsnorm(x, r, w, 1e-5)
        want, want_r = ref.fused_add_rmsnorm(x, r0, w, 1e-5)
        assert torch.equal(r, want_r)
        assert (out2.float() - want).abs().max().item() < 3e-2


def test_silu_mul():
    ops, ref = sub("ops"), sub("ops.reference")
    x = torch.randn(77, 2 * 1792, device="cuda").to(torch.bfloat16)
    assert (ops.silu_mul(x).float() - ref.silu_mul(x)).abs().max().item() < 3e-2


def test_rope_and_paged_cache_write():
    ops, ref = sub("ops"), sub("ops.reference")
    torch.manual_seed(0)
    T, nq, nkv, D, page = 50, 8, 2, 128, 16
    cs = ops.rope_cos_sin(4096, D, 500000.0, "cuda")
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda").to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), device="cuda", dtype=torch.int32)
    blocks = 8
    kc = torch.zeros(blocks, nkv, page, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(blocks * page, device="cuda")[:T].to(torch.int64)
    q = ops.rope_and_cache(qkv, pos, cs, nq, nkv, slots, kc, vc)
    q_ref = ref.rope(qkv[:, : nq * D].view(T, nq, D), pos, cs)
    k_ref = ref.rope(qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D), pos, cs)
    v_ref = qkv[:, (nq + nkv) * D:].view(T, nkv, D)
    assert (q.float() - q_ref).abs().max().item() < 3e-2
    blk, off = slots // page, slots % page
    assert (kc[blk, :, off, :].float() - k_ref).abs().max().item() < 3e-2
    assert torch.equal(vc[blk, :, off, :], v_ref)


def test_rope_with_qk_norm_and_paged_cache_write():
    """Qwen3's per-head q/k RMSNorm fused into the RoPE + cache-write kernel,
    against the fp32 reference: rope(rmsnorm(head) * w); v copied as is."""
    ops, ref = sub("ops"), sub("ops.reference")
    torch.manual_seed(1)
    T, nq, nkv, D, page, eps = 37, 16, 4, 128, 16, 1e-6
    cs = ops.rope_cos_sin(4096, D, 1000000.0, "cuda")
    qkv = (3 * torch.randn(T, (nq + 2 * nkv) * D, device="cuda")).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), device="cuda", dtype=torch.int32)
    qw = (1 + 0.3 * torch.randn(D, device="cuda")).to(torch.bfloat16)
    kw = (1 + 0.3 * torch.randn(D, device="cuda")).to(torch.bfloat16)
    blocks = 6
    kc = torch.zeros(blocks, nkv, page, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(blocks * page, device="cuda")[:T].to(torch.int64)
    q = ops.rope_and_cache(qkv, pos, cs, nq, nkv, slots, kc, vc, q_norm=qw, k_norm=kw, eps=eps)
    q_ref = ref.rope(ref.rmsnorm(qkv[:, :nq * D].view(T, nq, D), qw, eps), pos, cs)
    k_ref = ref.rope(ref.rmsnorm(qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D), kw, eps), pos, cs)
    # one bf16 rounding of values up to ~10: compare relative to the magnitude
    assert torch.allclose(q.float(), q_ref, rtol=1 / 128, atol=1e-2)
    blk, off = slots // page, slots % page
    assert torch.allclose(kc[blk, :, off, :].float(), k_ref, rtol=1 / 128, atol=1e-2)
    assert torch.equal(vc[blk, :, off, :], qkv[:, (nq + nkv) * D:].view(T, nkv, D))
    # without slots (no cache given) the kernel produces the same q
    q2 = ops.rope_and_cache(qkv, pos, cs, nq, nkv, q_norm=qw, k_norm=kw, eps=eps)
    assert torch.equal(q2, q)


def test_vocab_parallel_embedding():
    ops = sub("ops")
    table = torch.randn(1000, 256, device="cuda").to(torch.bfloat16)
    ids = torch.tensor([0, 999, 1000, 1500, 2999, 5], device="cuda", dtype=torch.int32)
    out = ops.embedding(ids, table, start=1000)  # shard holds ids [1000, 2000)
    assert torch.equal(out[2], table[0]) and torch.equal(out[3], table[500])
    assert out[0].abs().sum() == 0 and out[4].abs().sum() == 0


def test_argmax_and_combine():
    ops = sub("ops")
    torch.manual_seed(3)
    W, B, V = 4, 9, 5000
    logits = torch.randn(W, B, V, device="cuda").to(torch.bfloat16)
    vals, idxs = [], []
    for r in range(W):
        v, i = ops.argmax(logits[r], offset=r * V)
        vals.append(v)
        idxs.append(i)
    best = ops.argmax_combine(torch.stack(vals), torch.stack(idxs))
    full = logits.permute(1, 0, 2).reshape(B, W * V).float()
    assert torch.equal(best, full.argmax(-1))


def test_awq_int4_gemv_and_dequant():
    """AWQ int4 kernels against PyTorch: the dequantizer bit for bit (same
    fp32 product, one rounding), the GEMV (1..8 rows, with and without a
    residual) against x @ W^T in fp32."""
    ops, models = sub("ops"), sub("models")
    loader = sub("models.loader")
    torch.manual_seed(7)
    for N, K, G in ((512, 1024, 128), (1544, 512, 64), (64, 2048, 128)):
        wf = torch.randn(N, K) * 0.05
        qw, qz, s = models.awq_quantize(wf, G)
        w = ops.Int4Weight(qw.cuda(), qz.cuda(), s.cuda(), G)
        ref_w = loader.awq_dequant(qw, qz, s, G)                 # fp32 [N, K]
        assert torch.equal(ops.awq_dequant(w).cpu(), ref_w.to(torch.bfloat16))
        for M in (1, 3, 8):
            x = torch.randn(M, K).to(torch.bfloat16)
            want = x.float() @ ref_w.t()
            got = ops.awq_gemm(x.cuda(), w).float().cpu()
            tol = 2e-2 * want.abs().max().item() + 1e-2
            assert (got - want).abs().max().item() < tol, (N, K, G, M)
            res = torch.randn(M, N).to(torch.bfloat16)
            out = res.clone().cuda()
            ops.awq_gemm(x.cuda(), w, out=out, residual=out)       # in place, like the residual epilogue
            assert (out.float().cpu() - (want + res.float())).abs().max().item() < tol + 2e-2
        # 40 rows: the GEMV over 8-row chunks (row limit raised for the check)
        # and the dequant + tcgen05 GEMM path; 200 rows: the dequant path
        x = torch.randn(40, K).to(torch.bfloat16)
        want = x.float() @ ref_w.t()
        limit = ops.AWQ_GEMV_ROW_LIMIT
        for rows in (64, limit):
            ops.AWQ_GEMV_ROW_LIMIT = rows
            try:
                got = ops.awq_gemm(x.cuda(), w).float().cpu()
            finally:
                ops.AWQ_GEMV_ROW_LIMIT = limit
            assert (got - want).abs().max().item() < 2e-2 * want.abs().max().item() + 1e-2, rows
        x = torch.randn(200, K).to(torch.bfloat16)
        got = ops.awq_gemm(x.cuda(), w).float().cpu()
        want = x.float() @ ref_w.to(torch.bfloat16).float().t()
        assert (got - want).abs().max().item() < 2e-2 * want.abs().max().item() + 1e-2
