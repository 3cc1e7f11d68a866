"""tcgen05/TMEM GEMM vs a PyTorch fp32 reference (C = A @ B^T)."""
import pytest
import torch

from conftest import sub

pytestmark = pytest.mark.gpu

SHAPES = [
    # (M, N, K, bn, splits)
    (128, 256, 64, 256, 1),
    (128, 128, 128, 128, 1),
    (256, 512, 256, 0, 0),
    (200, 384, 320, 128, 1),      # M / N tails
    (1024, 4096, 4096, 0, 0),     # prefill o_proj at TP=1
    (1000, 3072, 4096, 0, 0),     # qkv at TP=2 with a ragged M
    (8, 6144, 4096, 0, 0),        # decode shape -> split-K
    (64, 1792, 14336, 0, 0),      # down_proj at TP=8 decode
    (1, 16032, 4096, 0, 0),       # lm_head shard, bs=1
    (96, 2048, 4096, 64, 1),      # BN=64 path
    (300, 960, 256, 160, 1),      # BN=160 with M/N tails
    (1024, 6144, 1024, 192, 1),   # BN=192
    (1024, 28672, 512, 224, 1),   # BN=224
    (130, 448, 640, 224, 1),      # BN=224 with tails
    (1, 768, 4096, 0, 0),         # swap-AB decode: TP=8 qkv, bs=1
    (33, 3584, 4096, 0, 0),       # swap-AB, 33 tokens (N side 64)
    (17, 4096, 512, 0, 0),        # swap-AB, short K
    (64, 4096, 1792, 0, 0),       # swap-AB, bs=64 TP=8 down
]


@pytest.mark.parametrize("M,N,K,bn,splits", SHAPES)
def test_gemm_matches_fp32(M, N, K, bn, splits):
    ops = sub("ops")
    torch.manual_seed(0)
    a = (torch.randn(M, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
    out = ops.gemm(a, w, bn=bn, splits=splits)
    torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    ref = a.float() @ w.float().t()
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale + 1e-2, f"max err {err} vs scale {scale}"


def test_gemm_swap_residual():
    """Decode-shaped GEMM (swap-AB path) with the residual add in the reduce."""
    ops = sub("ops")
    torch.manual_seed(4)
    M, N, K = 5, 4096, 2048
    a = (torch.randn(M, K, device="cuda") / 5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") / 5).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    out = ops.gemm(a, w, residual=r)
    ref = (a.float() @ w.float().t()).to(torch.bfloat16).float() + r.float()
    assert (out.float() - ref).abs().max().item() < 0.1


def test_gemm_residual_epilogue():
    ops = sub("ops")
    torch.manual_seed(1)
    M, N, K = 300, 1024, 512
    a = (torch.randn(M, K, device="cuda") / 5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") / 5).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    out = ops.gemm(a, w, residual=r)
    ref = (a.float() @ w.float().t()).to(torch.bfloat16).float() + r.float()
    assert (out.float() - ref).abs().max().item() < 0.1


@pytest.mark.parametrize("M", [1, 2, 3])
def test_gemv_rows_against_fp32(M):
    """1-2 rows run the CUDA-core GEMV (3 the tensor-core path, same check):
    fp32 accumulation of the bf16 stream, K slices that do not divide evenly
    among the warps, strided activations, and the residual form's two
    roundings."""
    ops = sub("ops")
    torch.manual_seed(10 + M)
    for N, K in ((1000, 4096), (24, 200), (6144, 4096), (4096, 14336)):
        big = (torch.randn(M, K + 64, device="cuda") / K ** 0.25).to(torch.bfloat16)
        a = big[:, :K]
        w = (torch.randn(N, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
        ref = a.float() @ w.float().t()
        out = ops.gemm(a, w)
        torch.cuda.synchronize()
        # one rounding of an fp32 sum: within a bf16 ulp plus accumulation-order noise
        assert (out.float() - ref).abs().max().item() <= 8e-3 * ref.abs().max().item() + 1e-3, (N, K)
        r = torch.randn(M, N, device="cuda").to(torch.bfloat16)
        got = ops.gemm(a, w, residual=r)
        want = ref.to(torch.bfloat16).float() + r.float()
        assert (got.float() - want).abs().max().item() < 0.1, (N, K)


def test_gemm_strided_views():
    """Operands that are row slices of bigger tensors (ld > K)."""
    ops = sub("ops")
    torch.manual_seed(2)
    big = (torch.randn(256, 1024, device="cuda") / 8).to(torch.bfloat16)
    a = big[:, :512]
    w = (torch.randn(384, 512, device="cuda") / 8).to(torch.bfloat16)
    out = ops.gemm(a, w)
    ref = a.float() @ w.float().t()
    assert (out.float() - ref).abs().max().item() < 2e-2 * ref.abs().max().item() + 1e-2


_PAIR_SCRIPT = r"""
import importlib, torch
ops = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops")
ref = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops.reference")
torch.manual_seed(0)
worst = 0.0
for (M, N, K, res) in [(256, 4096, 4096, False), (1024, 3072, 512, True), (589, 1000, 2048, False),
                       (2048, 6144, 4096, True), (1024, 28672, 1024, False), (300, 256, 64, True)]:
    a = (torch.randn(M, K, device="cuda") / 8).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") / 8).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda").to(torch.bfloat16) if res else None
    got = ops.gemm(a, w, residual=r).float()
    want = a.float() @ w.float().t()
    if res:
        want = want.to(torch.bfloat16).float() + r.float()
    err = ((got - want).abs() / (want.abs() + 1.0)).max().item()
    worst = max(worst, err)
    assert err < 2e-2, (M, N, K, res, err)
assert ops.gemm_error() == 0
print("PAIR-OK", worst)
"""


@pytest.mark.parametrize("pair_bn", ["256", "192", "128"])
def test_cta_pair_gemm_matches_reference(pair_bn):
    """The CTA-pair (cta_group::2) GEMM at each pair tile width, selected with
    MBX_GEMM_2CTA=1 and MBX_GEMM_2CTA_BN (read once per process, so it runs in
    a child), against the fp32 reference on ragged and multi-wave shapes,
    plain and residual epilogues."""
    import os
    import subprocess
    import sys

    env = dict(os.environ, MBX_GEMM_2CTA="1", MBX_GEMM_2CTA_BN=pair_bn)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT], env=env, cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0 and "PAIR-OK" in p.stdout, p.stdout[-2000:] + p.stderr[-4000:]


@pytest.mark.parametrize("M", [1, 2, 5])
def test_gemm_silu_matches_gemm_then_silu_mul(M):
    """The fused decode MLP input (one GEMV launch at 1-2 rows) rounds like the
    GEMM followed by silu_mul; 5 rows take that pair itself."""
    ops = sub("ops")
    torch.manual_seed(20 + M)
    for F, K in ((1792, 4096), (520, 1024)):
        x = (torch.randn(M, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
        w = (torch.randn(2 * F, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
        got = ops.gemm_silu(x, w)
        gu = ops.gemm(x, w)
        want = ops.silu_mul(gu)
        torch.cuda.synchronize()
        assert got.shape == (M, F)
        assert torch.equal(got, want), (F, K, (got.float() - want.float()).abs().max().item())


@pytest.mark.parametrize("M", [1, 2])
def test_qkv_rope_gemv_matches_gemm_then_rope(M):
    """The fused decode attention input (projection, neox RoPE, paged k/v
    writes in one GEMV launch) gives bit for bit what the GEMM followed by
    rope_and_cache gives."""
    ops = sub("ops")
    torch.manual_seed(30 + M)
    nq, nkv, K, page, blocks = 8, 2, 1024, 16, 6
    x = (torch.randn(M, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
    w = (torch.randn((nq + 2 * nkv) * 128, K, device="cuda") / K ** 0.25).to(torch.bfloat16)
    cos_sin = ops.rope_cos_sin(4096, 128, 10000.0, "cuda")
    pos = torch.tensor([37, 4000][:M], dtype=torch.int32, device="cuda")
    slots = torch.tensor([5 * page + 3, 2 * page + 15][:M], dtype=torch.int64, device="cuda")
    caches = [torch.zeros(blocks, nkv, page, 128, dtype=torch.bfloat16, device="cuda") for _ in range(4)]
    got_q = ops.qkv_rope_and_cache(x, w, pos, cos_sin, nq, nkv, slots, caches[0], caches[1])
    assert got_q is not None
    want_q = ops.rope_and_cache(ops.gemm(x, w), pos, cos_sin, nq, nkv, slots, caches[2], caches[3])
    torch.cuda.synchronize()
    assert torch.equal(got_q, want_q)
    assert torch.equal(caches[0], caches[2]) and torch.equal(caches[1], caches[3])
