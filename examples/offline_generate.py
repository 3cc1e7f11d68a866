"""Offline generation with the TP engine (one process per GPU):

    python examples/offline_generate.py --model tiny                          # random weights, 1 GPU
    python examples/offline_generate.py --model-path /path/to/Llama-3.1-8B --prompt "The capital of France is"
    SGLANG_MAILBOX_AR=1 torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/offline_generate.py --model 8b

Greedy by default; --temperature/--top-p/--top-k/--seed sample.
"""
import argparse
import importlib
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
PKG = "3080_mod_p2p_sglang_patch_b200"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", help="8b | 70b | tiny (random weights)")
    ap.add_argument("--model-path", default=None, help="Hugging Face checkpoint directory (Llama, Mistral, Qwen2/3)")
    ap.add_argument("--prompt", default="Hello from B200")
    ap.add_argument("--max-new", type=int, default=16)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-p", type=float, default=1.0)
    ap.add_argument("--top-k", type=int, default=0)
    ap.add_argument("--seed", type=int, default=None)
    args = ap.parse_args()
    par = importlib.import_module(f"{PKG}.parallel")
    models = importlib.import_module(f"{PKG}.models")
    eng_mod = importlib.import_module(f"{PKG}.engine")
    rank, world, local = par.init_distributed()
    dev = torch.device("cuda", local)
    tp = par.TPGroup(None, dev) if world > 1 else None  # MailboxAR when SGLANG_MAILBOX_AR=1, else NCCL
    if args.model_path:
        eng = eng_mod.LLMEngine.from_pretrained(args.model_path, tp=tp, device=dev, max_batch=4)
    else:
        eng = eng_mod.LLMEngine(models.LlamaConfig.by_name(args.model), tp=tp, device=dev, max_batch=4, max_seq=4096)
    out = eng.generate_text(args.prompt, {"max_new_tokens": args.max_new, "temperature": args.temperature,
                                          "top_k": args.top_k, "top_p": args.top_p, "seed": args.seed})
    if rank == 0:
        print(out)
    if eng.graphs is not None:
        eng.graphs.close()
    if tp is not None:
        tp.close()


if __name__ == "__main__":
    main()
