"""One rank of the multi-GPU allreduce suite (run under torchrun).

Mirrors the reference's hand-run scripts: bit-exact 2x smoke over varying
sizes (tests/test_mailbox_torch.py), graph capture + replays with changing
values (same file, :49-68, here 1000 replays), the 560-round hammer with a
per-round value (tests/hammer_mbx.py), and segmented-vs-full equality
(tests/hammer_seg.py); plus rank-distinct random inputs vs NCCL, the fused
allreduce+RMSNorm and the all-gather.
"""
import datetime
import importlib
import os
import sys

import torch
import torch.distributed as dist


def log(*a):
    if dist.get_rank() == 0:
        print(*a, flush=True)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel.communicator")
    cfg_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.config")
    cfg = cfg_mod.CommConfig.from_env()
    cfg.half_bytes = 16 << 20
    cfg.seg_slot_bytes = 2 << 20
    ar = comm_mod.MailboxAR(None, dev, config=cfg)
    assert not ar.disabled, "communicator did not come up"
    log(f"transport={ar.transport} world={world}")
    algos = ["oneshot_push", "oneshot_pull", "twoshot", "twoshot_push"] + (["nvls"] if "nvls" in ar.transport else [])

    # 1. bit-exact world*x with identical inputs on every rank, varying sizes
    torch.manual_seed(1234)
    for algo in algos:
        for it in range(40):
            nbytes = 4096 * (1 + (it * 37) % 300)
            x = torch.randn(nbytes // 2, dtype=torch.bfloat16, device=dev)
            out = ar.custom_all_reduce(x, algo=algo)
            want = (x.float() * world).to(torch.bfloat16)
            assert torch.equal(out, want), f"{algo} it{it} n={x.numel()} bad={(out != want).sum().item()}"
        torch.cuda.synchronize()
        assert ar.err() == 0
        log(f"bitexact {algo} OK")

    # 2. rank-distinct random inputs vs NCCL (fp32 / fp16 / bf16), chunked sizes too
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        for n in (8, 4096, 1 << 20, (40 << 20) // 4):
            g = torch.Generator(device=dev).manual_seed(100 + rank)
            x = torch.randn(n, device=dev, generator=g).to(dtype)
            for algo in algos:
                out = ar.custom_all_reduce(x, algo=algo)
                if out is None:
                    continue
                ref = x.float().clone()
                dist.all_reduce(ref)
                tol = 1e-5 if dtype == torch.float32 else 3e-2
                assert torch.allclose(out.float(), ref, rtol=tol, atol=tol * 4), f"{dtype} n={n} {algo}"
                # identical on every rank
                gathered = [torch.empty_like(out) for _ in range(world)]
                dist.all_gather(gathered, out)
                assert all(torch.equal(gathered[0], t) for t in gathered), f"ranks disagree {algo}"
    log("vs-NCCL OK")

    # 3. graph capture + 1000 replays with changing values
    n = (512 << 10) // 2
    x = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    for algo in algos:
        out = ar.custom_all_reduce(x, algo=algo)
        torch.cuda.synchronize()
        e0 = ar.epoch()
        g = torch.cuda.CUDAGraph()
        with ar.capture():
            with torch.cuda.graph(g):
                outg = ar.custom_all_reduce(x, algo=algo)
        for i in range(1000):
            x.fill_(float((i % 97) + 1) * 0.25)
            g.replay()
            if i % 250 == 0 or i == 999:
                torch.cuda.synchronize()
                assert torch.equal(outg, (x.float() * world).to(torch.bfloat16)), f"graph {algo} replay {i}"
        torch.cuda.synchronize()
        assert ar.epoch() == e0 + 1000, (ar.epoch(), e0)
        del g
    log("graph-1000 OK")

    # 4. hammer: 560 rounds, per-round value, three sizes (reference hammer_mbx.py)
    bad = 0
    for sz, iters in ((10 << 20, 300), (64 << 10, 200), (24575 << 10, 60)):
        for it in range(iters):
            v = (it % 251) + 1.0
            t = torch.full((sz // 2,), v, dtype=torch.bfloat16, device=dev)
            out = ar.custom_all_reduce(t)
            if not bool(torch.all(out.float() == world * v).item()):
                bad += 1
    assert bad == 0, f"hammer mismatches {bad}"
    log("hammer-560 OK")

    # 5. fused allreduce + residual + RMSNorm vs unfused
    ops_ref = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops.reference")
    for M, H in ((1, 4096), (64, 4096), (1024, 4096), (7, 8192)):
        g = torch.Generator(device=dev).manual_seed(7 + rank)
        xx = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
        res = torch.randn(M, H, device=dev, generator=torch.Generator(device=dev).manual_seed(9)).to(torch.bfloat16)
        w = torch.randn(H, device=dev, generator=torch.Generator(device=dev).manual_seed(11)).to(torch.bfloat16)
        for algo in (1, 3, 5):
            if algo == 1 and M * H * 2 > ar._ar.chunk_limit(1):
                continue  # one-shot slot is half_bytes / world
            r = res.clone()
            out = ar.all_reduce_rmsnorm(xx, r, w, 1e-5, algo=algo)
            s = ar.custom_all_reduce(xx, algo="twoshot")
            want, want_r = ops_ref.fused_add_rmsnorm(s, res, w, 1e-5)
            assert torch.equal(r, want_r), f"fused residual M={M} algo={algo}"
            assert (out.float() - want).abs().max().item() < 5e-2, f"fused norm M={M} algo={algo}"
    log("fused-rmsnorm OK")

    # 5b. fused row-parallel GEMM -> allreduce -> residual + RMSNorm, interleaved
    #     with plain allreduces (separate buffers/epochs must not interfere)
    for it, (M, K, N) in enumerate([(1, 512, 4096), (64, 1024, 4096), (1024, 2048, 4096), (333, 512, 8192)] * 25):
        g = torch.Generator(device=dev).manual_seed(1000 * rank + it)
        a = (torch.randn(M, K, device=dev, generator=g) / 8).to(torch.bfloat16)
        wt = (torch.randn(N, K, device=dev, generator=g) / 8).to(torch.bfloat16)
        gs = torch.Generator(device=dev).manual_seed(77 + it)  # same residual / norm weight on all ranks
        res = torch.randn(M, N, device=dev, generator=gs).to(torch.bfloat16)
        nw = (1 + 0.1 * torch.randn(N, device=dev, generator=gs)).to(torch.bfloat16)
        r = res.clone()
        out = ar.gemm_all_reduce_rmsnorm(a, wt, r, nw, 1e-5)
        plain = ar.custom_all_reduce(torch.full((4096,), float(rank), dtype=torch.bfloat16, device=dev))
        part = (a.float() @ wt.float().t()).to(torch.bfloat16).float()
        dist.all_reduce(part)
        want, want_r = ops_ref.fused_add_rmsnorm(part.to(torch.bfloat16), res, nw, 1e-5)
        assert (r.float() - want_r.float()).abs().max().item() < 0.05, f"fused gemm residual it={it}"
        assert (out.float() - want).abs().max().item() < 0.1, f"fused gemm out it={it}"
        assert torch.all(plain == float(sum(range(world)))), f"plain AR after fused it={it}"
        ga = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(ga, out)
        assert all(torch.equal(ga[0], t) for t in ga), "fused output differs across ranks"
    torch.cuda.synchronize()
    assert ar.err() == 0, ar.status()
    log("fused-gemm-allreduce OK")

    # 6. all-gather
    xg = torch.full((4096,), float(rank + 1), dtype=torch.bfloat16, device=dev)
    ag = ar.all_gather(xg)
    for r in range(world):
        assert torch.all(ag[r] == r + 1)
    log("allgather OK")

    # 7. segmented submit/wait == full allreduce, bit-exact (reference hammer_seg.py)
    side = ar.get_seg_stream()
    for rep in range(50):
        g = torch.Generator(device=dev).manual_seed(99 + rank * 1000 + rep)
        x = torch.randn(1024, 1024, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty_like(x)
        ev = torch.cuda.Event()
        ev.record()
        side.wait_event(ev)
        s1 = ar.submit_seg(x[:512], side)
        s2 = ar.submit_seg(x[512:], side)
        ar.wait_seg(s1, x[:512], out[:512])
        ar.wait_seg(s2, x[512:], out[512:])
        fb = ar.custom_all_reduce(x, algo="oneshot_push")
        torch.cuda.synchronize()
        assert ar.seg_err() == 0
        assert torch.equal(out, fb), f"seg rep {rep}"
    log("segmented OK")

    assert ar.err() == 0
    dist.barrier()
    ar.close()
    log("ALLREDUCE-SUITE-PASS")
    dist.destroy_process_group()


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        main()
    except BaseException:
        import traceback

        print(f"WORKER-ERROR rank {os.environ.get('RANK')}:\n{traceback.format_exc()}", flush=True)
        raise
