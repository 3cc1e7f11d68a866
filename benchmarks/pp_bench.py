"""Prompt-processing throughput through the HTTP server, measured the way the
reference's end-to-end benchmark does (tests/pp_bench.py): each request asks
for one token (``max_tokens=1``, so the time is the prefill), prompts differ
from the first token on (a prefix cache cannot serve them), and

    pp tok/s = usage.prompt_tokens / wall time of the request.

    python benchmarks/pp_bench.py --url http://127.0.0.1:8001                  # token-id prompts
    python benchmarks/pp_bench.py --text --sizes 131072,131072,40960,40960     # chat text (real tokenizer)

Token-id prompts (``/v1/completions`` with ``"prompt": [ids]``) give exact
lengths with any tokenizer, the byte tokenizer of random-weight models
included. ``--text`` sends chat messages of salted text through
``/v1/chat/completions`` like the reference, for servers with a checkpoint's
tokenizer; the lengths are then approximate (4 characters per token). The
first request warms the server up and is not counted. Prints one line per
request, then ``SUMMARY {json}``.
"""
import argparse
import json
import random
import time

import requests


def _ids_prompt(n: int, salt: int, vocab: int):
    rng = random.Random(salt)
    return [rng.randrange(1, vocab) for _ in range(n)]


def _text_prompt(n: int, salt: int) -> str:
    sent = f"Batch {salt}: tensor-parallel inference fuses kernels, overlaps communication and pages the KV cache. "
    return f"[{salt}] " + sent * (4 * n // len(sent) + 1)


def one(url: str, n: int, salt: int, text: bool, vocab: int, timeout: float):
    """(prompt tokens, wall seconds) of one max_tokens=1 request."""
    if text:
        body = {"messages": [{"role": "user", "content": _text_prompt(n, salt) + "\n\nReply: ok"}],
                "max_tokens": 1, "temperature": 0}
        path = "/v1/chat/completions"
    else:
        body = {"prompt": _ids_prompt(n, salt, vocab), "max_tokens": 1, "temperature": 0}
        path = "/v1/completions"
    t0 = time.perf_counter()
    r = requests.post(url + path, json=body, timeout=timeout)
    dt = time.perf_counter() - t0
    if r.status_code != 200:
        raise RuntimeError(f"HTTP {r.status_code}: {r.text[:300]}")
    return r.json()["usage"]["prompt_tokens"], dt


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--url", default="http://127.0.0.1:8001")
    ap.add_argument("--sizes", default="8000,8000,4000,4000", help="prompt tokens per timed request")
    ap.add_argument("--warmup", type=int, default=2000, help="prompt tokens of the untimed first request")
    ap.add_argument("--text", action="store_true", help="chat text prompts instead of token ids")
    ap.add_argument("--vocab", type=int, default=256, help="token-id range of id prompts (256: byte tokenizer)")
    ap.add_argument("--timeout", type=float, default=600.0)
    args = ap.parse_args(argv)
    sizes = [int(s) for s in args.sizes.split(",") if s]
    one(args.url, args.warmup, 0, args.text, args.vocab, args.timeout)
    res = {}
    for i, n in enumerate(sizes, start=1):
        pt, dt = one(args.url, n, i, args.text, args.vocab, args.timeout)
        res[f"{n}-{i}"] = {"prompt_tokens": pt, "wall_s": round(dt, 4), "pp_tok_s": round(pt / dt)}
        print(f"{n}-{i}: prompt={pt} wall={dt:.3f}s pp={pt / dt:.0f} tok/s", flush=True)
    total = sum(v["prompt_tokens"] for v in res.values())
    wall = sum(v["wall_s"] for v in res.values())
    print("SUMMARY " + json.dumps({"requests": res, "pp_tok_s_overall": round(total / wall) if wall else None}),
          flush=True)
    return res


if __name__ == "__main__":
    main()
