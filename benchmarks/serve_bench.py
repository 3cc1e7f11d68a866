"""Mixed serving: 70B-class decoder at TP = world size,
64 requests with uniform-random prompt lengths in [512, 8192] and 512
generated tokens each, served by the engine's own scheduler (chunked prefill
first, CUDA-graph decode batches otherwise).

    torchrun --nproc-per-node 8 benchmarks/serve_bench.py [--model 70b] [--impl native|torch]

Every engine step is device-timed with CUDA events (max over ranks). Reports
prefill tokens/s (prompt tokens / time in prefill steps), decode ITL p50/p99
(time per decode step) and the end-to-end wall time.
"""
import argparse
import importlib
import json
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="70b")
    ap.add_argument("--impl", default="native", choices=["native", "torch"])
    ap.add_argument("--int4", action="store_true", help="random weights packed as AWQ int4 (native only)")
    ap.add_argument("--mixed-chunk", action="store_true", help="prefill batches carry decode tokens")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--min-prompt", type=int, default=512)
    ap.add_argument("--max-prompt", type=int, default=8192)
    ap.add_argument("--gen", type=int, default=512)
    ap.add_argument("--chunk", type=int, default=8192)
    ap.add_argument("--sp", type=int, default=1, choices=[0, 1],
                    help="sequence-parallel prefill (fused GEMM->reduce-scatter, all-gather->GEMM); native only")
    args = ap.parse_args()
    par = importlib.import_module(f"{PKG}.parallel")
    models = importlib.import_module(f"{PKG}.models")
    eng_mod = importlib.import_module(f"{PKG}.engine")
    rank, world, local = par.init_distributed(timeout_s=900)
    dev = torch.device("cuda", local)
    tp = par.TPGroup(None, dev, use_mailbox=(args.impl == "native")) if world > 1 else None
    cfg = models.LlamaConfig.by_name(args.model)
    weights = None
    if args.int4:  # the random weights packed as AWQ int4 (int4 GEMV decode, per-layer expansion for prefill)
        weights = models.LlamaWeights(cfg, tp.rank if tp else 0, world, dev, seed=0)
        models.quantize_weights_int4(weights)
    eng = eng_mod.LLMEngine(cfg, tp=tp, max_batch=args.requests, max_seq=args.max_prompt + args.gen + 16,
                            chunk=args.chunk, seed=0, use_graphs=True, impl=args.impl,
                            sp=bool(args.sp) and args.impl == "native" and not args.int4,
                            mixed_chunk=args.mixed_chunk, weights=weights, device=dev)
    g = torch.Generator().manual_seed(11)
    lens = torch.randint(args.min_prompt, args.max_prompt + 1, (args.requests,), generator=g).tolist()
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in lens]
    # warm-up: capture graphs and touch every kernel once
    eng.generate([prompts[0][:128]], max_new_tokens=4)
    for p in prompts:
        eng.add_request(p, args.gen)
    pre_ms, dec_ms, pre_tok = 0.0, [], 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    wall0 = time.perf_counter()
    while eng.sched.has_work():
        e0.record()
        batch = eng.step()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if batch.kind == "prefill":
            pre_ms += ms
            pre_tok += batch.num_tokens
        else:
            dec_ms.append(ms)
    wall = time.perf_counter() - wall0
    t = torch.tensor([pre_ms, wall] + dec_ms, dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    pre_ms, wall = t[0].item(), t[1].item()
    dec = sorted(t[2:].tolist())
    if rank == 0:
        print(json.dumps({
            "metric": "mixed_serving", "model": cfg.name, "impl": args.impl, "tp": world, "requests": args.requests,
            "int4_weights": args.int4, "mixed_chunk": args.mixed_chunk,
            "sequence_parallel": eng.sp is not None,
            "prompt_tokens": pre_tok, "gen_tokens": args.requests * args.gen,
            "prefill_tok_s": pre_tok / (pre_ms * 1e-3),
            "decode_itl_p50_ms": dec[len(dec) // 2] if dec else None,
            "decode_itl_p99_ms": dec[min(len(dec) - 1, int(len(dec) * 0.99))] if dec else None,
            "decode_steps": len(dec), "wall_s": wall,
            "total_tok_s": (pre_tok + args.requests * args.gen) / wall,
        }), flush=True)
    if eng.graphs is not None:
        eng.graphs.close()
    if tp is not None:
        tp.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
