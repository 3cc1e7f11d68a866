"""Perplexity of a text through the engine (prompt scoring, the same path as
the server's ``echo`` logprobs): a whole-model accuracy check.

    python benchmarks/perplexity.py --model-path /path/to/ckpt --text corpus.txt
    python benchmarks/perplexity.py --model tiny --tokens 2048 --impl native --compare oracle

The text is cut into windows of ``--window`` tokens, scored one window per
request; every token but a window's first contributes -log p(token | the
window's tokens before it). ``--compare IMPL`` scores the same windows with a
second build of the same weights (``oracle``: the fp32 restatement of every
kernel) and reports both perplexities and the mean absolute difference of
the per-token logprobs. ``--int4-weights`` keeps an AWQ checkpoint packed.
Prints one JSON line.
"""
import argparse
import importlib
import json
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
PKG = "3080_mod_p2p_sglang_patch_b200"


def score(eng, windows):
    """Per-token logprobs of every window (first token of each excluded)."""
    out = []
    for w in windows:
        r = eng.add_request(w, 1, prompt_logprobs=True)
        eng.run()
        out.extend(v for v, _ in r.prompt_token_logprobs[1:])
    return out


def build(args, impl, device, weights=None):
    models = importlib.import_module(f"{PKG}.models")
    eng_mod = importlib.import_module(f"{PKG}.engine")
    kw = dict(max_batch=2, chunk=args.chunk, use_graphs=False, impl=impl, max_seq=args.window + 8)
    if args.model_path:
        if weights is not None:
            cfg = weights[0]
            return eng_mod.LLMEngine(cfg, device=device, weights=weights[1], **kw)
        return eng_mod.LLMEngine.from_pretrained(args.model_path, device=device, int4_weights=args.int4_weights,
                                                 **kw)
    cfg = models.LlamaConfig.by_name(args.model)
    return eng_mod.LLMEngine(cfg, device=device, seed=args.seed, full_init=True, **kw)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="tiny", help="8b | 70b | tiny (random weights)")
    ap.add_argument("--model-path", default=None)
    ap.add_argument("--text", default=None, help="a text file (needs a checkpoint tokenizer), else random ids")
    ap.add_argument("--tokens", type=int, default=2048, help="random token ids to score without --text")
    ap.add_argument("--window", type=int, default=1024)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--impl", default="native", choices=["native", "torch", "oracle"])
    ap.add_argument("--compare", default=None, choices=["native", "torch", "oracle"])
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--int4-weights", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    eng = build(args, args.impl, args.device)
    if args.text:
        if eng.tokenizer is None:
            raise SystemExit("--text needs a checkpoint with a tokenizer")
        with open(args.text) as f:
            ids = eng.tokenizer.encode(f.read())
    else:
        g = torch.Generator().manual_seed(args.seed)
        ids = torch.randint(0, eng.cfg.vocab, (args.tokens,), generator=g).tolist()
    windows = [ids[i:i + args.window] for i in range(0, len(ids), args.window) if len(ids[i:i + args.window]) > 1]
    lp = score(eng, windows)
    res = {"bench": "perplexity", "model": eng.cfg.name, "impl": args.impl, "tokens": len(lp),
           "nll": -sum(lp) / len(lp), "ppl": math.exp(-sum(lp) / len(lp))}
    if args.compare:
        other = build(args, args.compare, args.device, weights=(eng.cfg, eng.weights) if args.model_path else None)
        lp2 = score(other, windows)
        res.update({"compare": args.compare, "ppl_compare": math.exp(-sum(lp2) / len(lp2)),
                    "mean_abs_logprob_diff": sum(abs(a - b) for a, b in zip(lp, lp2)) / len(lp)})
    print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()
