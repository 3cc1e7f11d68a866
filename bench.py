"""Headline benchmark: tensor-parallel prefill tokens/s of the Llama-style 8B
decoder (hidden 4096, 32 layers, 32q/8kv heads, FFN 14336,
vocab 128256, bf16, random-init weights N(0, 0.02); 16 requests x 4096
uniform-random token ids, chunked prefill with chunk 1024), TP = --gpus.

    python bench.py --gpus N --steps K --warmup W [--impl native|torch|reference]

One step = the whole prefill of the 16 x 4096 batch (64 chunk forwards).
``value`` is device-timed (CUDA events, barrier + synchronize on both sides,
max over ranks) with the chunk inputs already on the device; ``e2e`` runs the
same prefill through the public API ``LLMEngine.generate(prompts,
max_new_tokens=1)`` (the reference's pp-bench shape, tests/pp_bench.py),
whose timed region includes the pinned host->device copies of every chunk's
inputs and the device->host read of the generated tokens.

--impl torch   : this repo's NCCL(+cuBLAS) TP build (F.linear + NCCL allreduce).
--impl reference : the unmodified reference; it ships no model, engine or
                   packaging, so the metric cannot be measured through it.
Multi-GPU: launch with torch.distributed.run (one rank per GPU).
"""
import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "3080_mod_p2p_sglang_patch_b200"

# The reference's only published prefill number (chunk 1024, 40K prompt):
# reference docs/performance.md:43. It was taken on 2x RTX 3080 with a 27B
# AWQ-int4 model at TP=2, so no ratio to it is printed (``vs_baseline`` is
# null); it is carried in ``config`` as context only.
REFERENCE_PUBLISHED_PREFILL_TOKS = 1464.0

REFERENCE_UNAVAILABLE = (
    "the reference (ackerx/3080_mod_p2p_sglang_patch) is an allreduce plugin for sglang 0.5.19 with no model, "
    "engine or packaging (pip: 'neither setup.py nor pyproject.toml found'); sglang is not installed and cannot be "
    "built offline, so prefill tok/s cannot be measured through its public API")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "torch", "reference"])
    p.add_argument("--model", default="8b")
    p.add_argument("--requests", type=int, default=16)
    p.add_argument("--prompt-len", type=int, default=4096)
    p.add_argument("--chunk", type=int, default=1024)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--sp", type=int, default=None, choices=[0, 1],
                   help="sequence-parallel prefill (1) or allreduce prefill (0); default: MBX_SP (off)")
    p.add_argument("--overlap", type=int, default=None, choices=[0, 1],
                   help="overlapped micro-batches at TP > 1 (1) or one batch per chunk (0); default: MBX_OVERLAP")
    p.add_argument("--no-graph", action="store_true", help="launch every chunk's kernels eagerly (the torch "
                   "baseline always does: like sglang, it graphs decode only)")
    return p.parse_args()


def main():
    args = parse()
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE}))
        return 0

    import importlib

    import torch
    import torch.distributed as dist

    par = importlib.import_module(f"{PKG}.parallel")
    models = importlib.import_module(f"{PKG}.models")
    eng_mod = importlib.import_module(f"{PKG}.engine")
    ops = importlib.import_module(f"{PKG}.ops")
    launches = importlib.import_module(f"{PKG}.utils.launches")
    utils = importlib.import_module(f"{PKG}.utils")

    rank, world, local = par.init_distributed(timeout_s=300)
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tp = par.TPGroup(None, dev, use_mailbox=(args.impl == "native")) if world > 1 else None

    cfg = models.LlamaConfig.by_name(args.model)
    R, S, chunk = args.requests, args.prompt_len, args.chunk
    eng = eng_mod.LLMEngine(cfg, tp=tp, max_batch=R, max_seq=S + 16, chunk=chunk, seed=0, use_graphs=False,
                            impl=args.impl, prefill_graph=(args.impl == "native" and not args.no_graph),
                            sp=(None if args.sp is None else bool(args.sp)) if args.impl == "native" else False,
                            overlap=None if args.overlap is None else bool(args.overlap))
    g = torch.Generator().manual_seed(1234)
    prompts = torch.randint(0, cfg.vocab, (R, S), generator=g).tolist()

    # ---- device-timed path: the exact chunk sequence of the scheduler, inputs staged on the device
    reqs = [eng.add_request(p, 1) for p in prompts]
    plan = []
    while eng.sched.prefilling or eng.sched.waiting:
        b = eng.sched.next_batch()
        for p in b.pieces:
            if not getattr(p.req, "_row_synced", False):
                eng._sync_block_row(p.req)
        # capture (request, start, n, blocks, table row) before the scheduler retires the request
        plan.append([(p.req, p.start, p.n, list(p.req.blocks), p.req.slot) for p in b.pieces])
        eng.sched.after_prefill(b, [0] * len(b.pieces))
    eng.sched.finished.clear()
    staged = []
    for pieces in plan:
        ids, pos, slots, q_lens, kv_lens, rows, last = [], [], [], [], [], [], []
        off = 0
        for rq, start, n, blocks, row in pieces:
            ids += rq.prompt[start:start + n]
            pos += list(range(start, start + n))
            slots += eng.kv.slots(blocks, start, n)
            q_lens.append(n)
            kv_lens.append(start + n)
            rows.append(row)
            off += n
            last.append(off - 1)
        cu = [0]
        for q in q_lens:
            cu.append(cu[-1] + q)
        st = {
            "ids": torch.tensor(ids, dtype=torch.int32, device=dev),
            "pos": torch.tensor(pos, dtype=torch.int32, device=dev),
            "slots": torch.tensor(slots, dtype=torch.int64, device=dev),
            "cu": torch.tensor(cu, dtype=torch.int32, device=dev),
            "kvl": torch.tensor(kv_lens, dtype=torch.int32, device=dev),
            "bt": eng.block_table.index_select(0, torch.tensor(rows, device=dev)),
            "tiles": ops.prefill_tiles(q_lens).to(dev),
            "last": torch.tensor(last, dtype=torch.int64, device=dev),
            "splits": ops.prefill_splits(len(ops.prefill_tiles(q_lens)), cfg.heads // world, max(kv_lens)),
            "graph": len(pieces) == 1 and q_lens[0] == chunk,
            "kv_int": kv_lens[0],
        }
        staged.append(st)
    tokens_per_step = sum(sum(n for _, _, n, _, _ in pieces) for pieces in plan)
    scale = eng.model.scale

    def run_step():
        out = None
        for st in staged:
            if eng.prefill_graph is not None and st["graph"]:
                out = eng.prefill_graph.run(st["ids"], st["pos"], st["slots"], st["kv_int"], st["bt"][0])
                continue

            def attn(li, q, kc, vc, st=st):
                return ops.prefill_attention(q, kc, vc, st["cu"], st["kvl"], st["bt"], st["tiles"], scale,
                                             splits=st["splits"])
            out = eng.model.forward(st["ids"], st["pos"], st["slots"], eng.kv.caches, attn, st["last"])
        return out

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    launches.reset()
    sampler = utils.ClockSampler(None if world > 1 else local) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    with utils.DeviceTimer() as t:
        for _ in range(args.steps):
            run_step()
    if sampler:
        sampler.__exit__(None, None, None)
    n_launch = launches.get()
    ms_per_step = t.max_ms / args.steps
    value = tokens_per_step / (ms_per_step / 1e3)

    # ---- end-to-end through the public API (fresh requests every step)
    e2e = None
    if not args.no_e2e:
        eng.generate(prompts[:2], max_new_tokens=1)  # warm the host path
        bi = tokens_per_step * (4 + 4 + 8) + len(plan) * 64  # ids+pos (int32) + slots (int64) + per-chunk metadata
        bo = R * 8  # one int64 token per request
        walls = []
        for _ in range(max(1, args.steps)):
            utils.timing.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            outs = eng.generate(prompts, max_new_tokens=1)
            torch.cuda.synchronize()
            walls.append(time.perf_counter() - t0)
            assert len(outs) == R and all(len(o) == 1 for o in outs)
        wall = utils.max_over_ranks(sorted(walls)[len(walls) // 2])
        e2e = {"value": tokens_per_step / wall, "unit": "tokens/s", "h2d_bytes_per_step": bi,
               "d2h_bytes_per_step": bo}

    clocks = sampler.summary() if sampler else None
    if rank == 0:
        line = {
            "metric": "prefill_tokens_per_s",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform-random token ids, random-init weights N(0,0.02))",
            "impl": args.impl,
            "config": {
                "model": cfg.name, "global_batch": R, "seq_len": S, "chunk": chunk,
                "parallelism": f"tp{world}",
                "l2": "no flush: weights (16 GB) and KV cache (8 GB) exceed the 126 MB L2 every step",
                "baseline_context": f"{REFERENCE_PUBLISHED_PREFILL_TOKS:.0f} tok/s, reference docs/performance.md:43 "
                                    "(2x RTX 3080, 27B AWQ-int4, TP=2): other hardware and model, not a ratio",
                "transport": getattr(tp.ca_comm, "transport", None) if (tp and tp.ca_comm) else None,
                "prefill_cuda_graph": eng.prefill_graph is not None,
                "sequence_parallel": eng.sp is not None,
                "overlapped_micro_batches": bool(eng.overlap),
                "gemm_cta_pair": {"0": "off", "1": "on"}.get(os.environ.get("MBX_GEMM_2CTA", ""), "by wave cost"),
                "fused_gemm_allreduce": bool(tp is not None and tp.fused_gemm_ar),
            },
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")} if clocks else None,
            "e2e": e2e,
            "gpu_launches": n_launch,
        }
        print(json.dumps(line), flush=True)
    if tp is not None:
        tp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
