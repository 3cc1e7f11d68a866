"""CUDA-graph decode ITL: Llama-style 8B at TP = world
size, batch sizes {1, 8, 32, 64}, every request with a 4096-token
uniform-random-id context prefilled into the paged KV cache (page 16, bf16),
then 256 tokens generated greedily.

    torchrun --nproc-per-node N benchmarks/decode_bench.py [--impl native|torch]

Each decode step replays the batch size's captured graph; its device time is
taken with CUDA events around the replay (max over ranks). Reports ITL p50/p99
(ms) and decode tokens/s per batch size as JSON lines.
"""
import argparse
import importlib
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="8b")
    ap.add_argument("--impl", default="native", choices=["native", "torch"])
    ap.add_argument("--int4", action="store_true", help="random weights packed as AWQ int4 (native only)")
    ap.add_argument("--batches", default="1,8,32,64")
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--gen", type=int, default=256)
    args = ap.parse_args()
    par = importlib.import_module(f"{PKG}.parallel")
    models = importlib.import_module(f"{PKG}.models")
    eng_mod = importlib.import_module(f"{PKG}.engine")
    utils = importlib.import_module(f"{PKG}.utils")
    rank, world, local = par.init_distributed(timeout_s=600)
    dev = torch.device("cuda", local)
    tp = par.TPGroup(None, dev, use_mailbox=(args.impl == "native")) if world > 1 else None
    cfg = models.LlamaConfig.by_name(args.model)
    batches = [int(b) for b in args.batches.split(",")]
    max_bs = max(batches)
    weights = None
    if args.int4:  # the random weights packed as AWQ int4 (int4 GEMV decode)
        weights = models.LlamaWeights(cfg, tp.rank if tp else 0, world, dev, seed=0)
        models.quantize_weights_int4(weights)
    eng = eng_mod.LLMEngine(cfg, tp=tp, max_batch=max_bs, max_seq=args.ctx + args.gen + 16, chunk=8192, seed=0,
                            use_graphs=True, impl=args.impl, graph_sizes=tuple(sorted(set(batches))),
                            weights=weights, device=dev)
    g = torch.Generator().manual_seed(7)
    for bs in batches:
        prompts = torch.randint(0, cfg.vocab, (bs, args.ctx), generator=g).tolist()
        reqs = [eng.add_request(p, args.gen) for p in prompts]
        # prefill everything first
        while eng.sched.prefilling or eng.sched.waiting:
            eng.step()
        times = []
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = 0
        while eng.sched.running:
            batch = eng.sched.next_batch()
            for r in batch.reqs:
                if not getattr(r, "_row_synced", False):
                    eng._sync_block_row(r)
            ids, pos, kv_len, slots, rows = eng.decode_inputs(batch.reqs)
            if eng.graphs is not None and not eng.graphs._captured:
                eng.graphs.capture()
            torch.cuda.synchronize()
            e0.record()
            out = eng.graphs.run(ids, pos, kv_len, slots, rows)
            e1.record()
            nxt = out.tolist()
            times.append(e0.elapsed_time(e1))
            eng.sched.after_decode(batch, nxt)
            steps += 1
        eng.sched.finished.clear()
        t = torch.tensor(times, dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ts = sorted(t.tolist()[3:])  # first replays include lazy work
        p50 = ts[len(ts) // 2]
        p99 = ts[min(len(ts) - 1, int(len(ts) * 0.99))]
        mean = sum(ts) / len(ts)
        if rank == 0:
            print(json.dumps({"metric": "decode_itl", "model": cfg.name, "impl": args.impl, "tp": world, "batch": bs,
                              "int4_weights": args.int4,
                              "ctx": args.ctx, "gen": args.gen, "itl_p50_ms": p50, "itl_p99_ms": p99,
                              "decode_tok_s": bs / (mean * 1e-3), "steps": steps}), flush=True)
    if eng.graphs is not None:
        eng.graphs.close()
    if tp is not None:
        tp.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
