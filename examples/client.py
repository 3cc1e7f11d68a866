"""Client for the OpenAI-compatible server (start it with
``torchrun ... -m 3080_mod_p2p_sglang_patch_b200.server``):

    python examples/client.py --url http://127.0.0.1:8001 --prompt "hi" [--stream] [--temperature 0.7]

Prints the completion, then the prompt-processing rate measured the way the
reference's benchmark does (usage.prompt_tokens / wall time, max_tokens=1).
"""
import argparse
import json
import time

import requests


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", default="http://127.0.0.1:8001")
    ap.add_argument("--prompt", default="Explain NVLink in one sentence.")
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--stream", action="store_true")
    args = ap.parse_args(argv)
    body = {"messages": [{"role": "user", "content": args.prompt}], "max_tokens": args.max_tokens,
            "temperature": args.temperature, "stream": args.stream}
    if args.stream:
        with requests.post(args.url + "/v1/chat/completions", json=body, stream=True, timeout=600) as r:
            for line in r.iter_lines(decode_unicode=True):
                if line.startswith("data: ") and line != "data: [DONE]":
                    chunk = json.loads(line[6:])
                    print(chunk["choices"][0].get("delta", {}).get("content", ""), end="", flush=True)
        print()
    else:
        j = requests.post(args.url + "/v1/chat/completions", json=body, timeout=600).json()
        print(j["choices"][0]["message"]["content"], j["usage"])
    body.update(max_tokens=1, stream=False, messages=[{"role": "user", "content": args.prompt * 200}])
    t0 = time.time()
    j = requests.post(args.url + "/v1/chat/completions", json=body, timeout=600).json()
    dt = time.time() - t0
    print(f"prompt={j['usage']['prompt_tokens']} tokens in {dt:.3f}s -> {j['usage']['prompt_tokens'] / dt:.0f} tok/s")


if __name__ == "__main__":
    main()
