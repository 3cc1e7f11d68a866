"""The communicator's cross-rank kernels on ONE GPU, every rank emulated.

``parallel.emulate.EmulatedWorld`` runs all W ranks' blocks of a call in one
cooperative launch (the only way ranks that wait on one another may share a
GPU), each rank with its own buffers, state and status words. The device code
is the multi-GPU code; only the peers' memory is local. Every result is
checked against a plain PyTorch fp32 reference:

* allreduce (one-shot push / pull, two-shot, two-shot push; bf16 and fp32):
  bit-exact against the fp32 sum in rank order with one final rounding, over
  consecutive calls with new values (ping-pong halves and epochs move on);
* allreduce + residual + RMSNorm (one-shot push, two-shot, two-shot push),
  with 512- and 256-thread blocks (the latter is the overlapped prefill's);
* the fused row-parallel GEMM -> allreduce -> residual + RMSNorm (push-all
  and owner-push epilogues);
* all-gather.

The reference runs its protocol tests on two real GPUs only
(tests/test_mailbox_torch.py:34-68, tests/hammer_mbx.py:24-38).
"""
import pytest
import torch

from conftest import sub

pytestmark = pytest.mark.gpu

ALGOS = ["oneshot_push", "oneshot_pull", "twoshot", "twoshot_push"]


def _world(W, **kw):
    return sub("parallel.emulate").EmulatedWorld(W, **kw)


def _rank_sum(xs):
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()
    return acc


def _rand(shape, seed, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_emulated_allreduce_bit_exact(W, dtype):
    comm = sub("parallel.communicator")
    with _world(W) as ew:
        calls = 0
        for algo in ALGOS:
            a = comm.ALGO_IDS[algo]
            # sizes: one vector, ragged against blocks and chunks, 0.5-1 MB
            # (one launch: the one-shot slot is half / W = 1 MB at W = 8)
            for numel in (8, 4096 * 3 + 40, 1 << 18):
                for rep in range(2):
                    xs = [_rand((numel,), 1000 * calls + 17 * r + rep, dtype) for r in range(W)]
                    want = _rank_sum(xs).to(dtype)
                    # the second repetition reduces in place (out == in)
                    outs = ew.allreduce(xs, algo=a, outs=xs if rep else None)
                    torch.cuda.synchronize()
                    ew.check()
                    for r in range(W):
                        assert torch.equal(outs[r], want), f"{algo} numel={numel} rank {r}"
                    calls += 1
        assert ew.epochs() == [calls] * W


@pytest.mark.parametrize("threads", [512, 256])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_emulated_allreduce_rmsnorm(W, threads):
    comm, ref = sub("parallel.communicator"), sub("ops.reference")
    H, eps = 1024, 1e-5
    w = (1.0 + 0.1 * _rand((H,), 3)).to(torch.bfloat16)
    with _world(W) as ew:
        for algo in ("oneshot_push", "twoshot", "twoshot_push"):
            for M in (1, 7, 64, 300):
                xs = [_rand((M, H), 100 * M + r) for r in range(W)]
                res0 = _rand((M, H), 7 + M)
                residuals = [res0.clone() for _ in range(W)]
                outs = ew.all_reduce_rmsnorm(xs, residuals, w, eps, algo=comm.ALGO_IDS[algo], threads=threads)
                ar = _rank_sum(xs).to(torch.bfloat16)
                want_out, want_res = ref.fused_add_rmsnorm(ar, res0, w, eps)
                torch.cuda.synchronize()
                ew.check()
                for r in range(W):
                    assert torch.equal(residuals[r], want_res), f"{algo} M={M} rank {r}: residual"
                    err = (outs[r].float() - want_out).abs().max().item()
                    assert err < 3e-2, f"{algo} M={M} rank {r}: norm err {err}"


@pytest.mark.parametrize("push_all", [True, False])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_emulated_fused_gemm_allreduce_rmsnorm(W, push_all):
    ref = sub("ops.reference")
    K, N, eps = 512, 1024, 1e-5
    w_norm = (1.0 + 0.1 * _rand((N,), 5)).to(torch.bfloat16)
    with _world(W, fuse_half_bytes=16 << 20) as ew:
        for M in (64, 200, 513):
            a_s = [_rand((M, K), 300 + r) for r in range(W)]
            w_s = [(_rand((N, K), 400 + r) * 0.05).to(torch.bfloat16) for r in range(W)]
            res0 = _rand((M, N), 11)
            residuals = [res0.clone() for _ in range(W)]
            outs = ew.gemm_all_reduce_rmsnorm(a_s, w_s, residuals, w_norm, eps, push_all=push_all)
            parts = [ref.gemm(a_s[r], w_s[r]).to(torch.bfloat16) for r in range(W)]
            ar = _rank_sum(parts).to(torch.bfloat16)
            want_out, want_res = ref.fused_add_rmsnorm(ar, res0, w_norm, eps)
            torch.cuda.synchronize()
            ew.check()
            assert int(ew.err.item()) == 0
            for r in range(W):
                # the tensor-core partials differ from fp32 matmul by accumulation order
                torch.testing.assert_close(residuals[r].float(), want_res.float(), rtol=2e-2, atol=2e-2,
                                           msg=lambda m: f"M={M} rank {r}: residual: {m}")
                assert torch.equal(residuals[r], residuals[0]), f"M={M}: ranks disagree"
                err = (outs[r].float() - want_out).abs().max().item()
                assert err < 6e-2, f"M={M} rank {r}: norm err {err}"


@pytest.mark.parametrize("W", [2, 8])
def test_emulated_allgather(W):
    with _world(W) as ew:
        for numel in (8, 4096 + 8):
            xs = [_rand((numel,), 50 + r) for r in range(W)]
            outs = ew.all_gather(xs)
            torch.cuda.synchronize()
            ew.check()
            want = torch.stack(xs)
            for r in range(W):
                assert torch.equal(outs[r], want)


def test_emulated_mixed_calls_share_epochs():
    """Allreduce, allreduce+norm and all-gather advance one epoch counter;
    interleaving them must keep every call's data apart (ping-pong halves)."""
    comm = sub("parallel.communicator")
    W, H = 4, 1024
    w = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    with _world(W) as ew:
        for it in range(12):
            v = float(it % 251 + 1)
            xs = [torch.full((64, H), v, dtype=torch.bfloat16, device="cuda") for _ in range(W)]
            outs = ew.allreduce(xs, algo=comm.ALGO_IDS[ALGOS[it % len(ALGOS)]])
            res = [torch.zeros(64, H, dtype=torch.bfloat16, device="cuda") for _ in range(W)]
            algo = comm.ALGO_TWOSHOT_PUSH if it % 2 else comm.ALGO_ONESHOT_PUSH
            ew.all_reduce_rmsnorm(xs, res, w, 1e-5, algo=algo)
            torch.cuda.synchronize()
            ew.check()
            want = torch.bfloat16
            for r in range(W):
                assert torch.all(outs[r] == torch.tensor(W * v, dtype=want, device="cuda"))
                assert torch.all(res[r] == torch.tensor(W * v, dtype=want, device="cuda"))
        assert ew.epochs() == [24] * W


_PAIR_PUSH_SCRIPT = r"""
import importlib, sys, torch
emulate = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel.emulate")
ref = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops.reference")
g = torch.Generator(device="cuda").manual_seed(7)
def rnd(*s):
    return torch.randn(*s, generator=g, device="cuda").to(torch.bfloat16)
K, N, eps = 1024, 2048, 1e-5
w_norm = torch.ones(N, dtype=torch.bfloat16, device="cuda")
worst = 0.0
for W, push_all in ((2, True), (4, False), (8, False)):
    with emulate.EmulatedWorld(W, fuse_half_bytes=24 << 20) as ew:
        for M in (512, 777):
            a_s = [rnd(M, K) for _ in range(W)]
            w_s = [(rnd(N, K) * 0.03).to(torch.bfloat16) for _ in range(W)]
            res0 = rnd(M, N)
            res = [res0.clone() for _ in range(W)]
            outs = ew.gemm_all_reduce_rmsnorm(a_s, w_s, res, w_norm, eps, push_all=push_all)
            parts = [ref.gemm(a_s[r], w_s[r]).to(torch.bfloat16).float() for r in range(W)]
            acc = parts[0].clone()
            for p in parts[1:]:
                acc += p
            want, _ = ref.fused_add_rmsnorm(acc.to(torch.bfloat16), res0, w_norm, eps)
            torch.cuda.synchronize()
            ew.check()
            assert int(ew.err.item()) == 0
            for r in range(W):
                assert torch.equal(res[r], res[0])
                err = (outs[r].float() - want).abs().max().item()
                worst = max(worst, err)
                assert err < 6e-2, (W, push_all, M, r, err)
print("PAIR-PUSH-OK", worst)
"""


@pytest.mark.parametrize("pair_bn", ["256", "192", "128"])
def test_emulated_fused_gemm_on_cta_pair_kernel(pair_bn):
    """The push epilogue on the CTA-pair GEMM (forced with MBX_GEMM_2CTA=1 and
    each pair tile width; read once per process, so it runs in a child):
    push-all at 2 ranks, owner push at 4 and 8, against fp32."""
    import os
    import subprocess
    import sys

    from conftest import ROOT

    env = dict(os.environ, MBX_GEMM_2CTA="1", MBX_GEMM_2CTA_BN=pair_bn)
    p = subprocess.run([sys.executable, "-c", _PAIR_PUSH_SCRIPT], env=env, cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0 and "PAIR-PUSH-OK" in p.stdout, p.stdout[-2000:] + p.stderr[-4000:]
