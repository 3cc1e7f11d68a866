"""Online serving benchmark against the HTTP server (the role of sglang's
``bench_serving``): many streamed requests, each timed by the client.

    python benchmarks/bench_serving.py --url http://127.0.0.1:8001 --num-requests 256 --concurrency 64 \
        --input-len 512:4096 --output-len 128

Each request is a ``/v1/completions`` call with a random token-id prompt (no
shared prefix) and ``stream: true``; arrivals follow ``--request-rate``
(Poisson, requests/s; inf = all at once) under a cap of ``--concurrency``
requests in flight. Per request the client records the time to the first
streamed token (TTFT), the gaps between later chunks (ITL, divided by the
tokens in the chunk) and the end-to-end latency. Prints one JSON line:
request and token throughput plus p50 / p90 / p99 of TTFT, ITL and latency.
"""
import argparse
import json
import random
import threading
import time


def _pct(xs, q):
    if not xs:
        return None
    v = sorted(xs)
    return v[min(len(v) - 1, int(q * len(v)))]


def one_request(url, prompt, max_tokens, timeout):
    """(ttft s, [per-token gaps s], latency s, output tokens) of one streamed request."""
    import requests

    body = {"prompt": prompt, "max_tokens": max_tokens, "stream": True, "temperature": 0}
    t0 = time.perf_counter()
    ttft, gaps, n_out, last = None, [], 0, None
    with requests.post(url + "/v1/completions", json=body, stream=True, timeout=timeout) as r:
        r.raise_for_status()
        for line in r.iter_lines(decode_unicode=True):
            if not line.startswith("data: ") or line == "data: [DONE]":
                continue
            chunk = json.loads(line[6:])
            if "error" in chunk:
                raise RuntimeError(chunk["error"])
            k = len(chunk["choices"][0].get("token_ids") or [])
            if k == 0:
                continue
            now = time.perf_counter()
            if ttft is None:
                ttft = now - t0
            else:
                gaps.extend([(now - last) / k] * k)
            last = now
            n_out += k
    return ttft, gaps, time.perf_counter() - t0, n_out


def run(url, num_requests, concurrency, request_rate, input_len, output_len, vocab, seed, timeout=600.0):
    rng = random.Random(seed)
    lo, hi = input_len
    prompts = [[rng.randrange(1, vocab) for _ in range(rng.randint(lo, hi))] for _ in range(num_requests)]
    arrivals, t = [], 0.0
    for _ in range(num_requests):
        arrivals.append(t)
        if request_rate != float("inf"):
            t += rng.expovariate(request_rate)
    sem = threading.Semaphore(concurrency)
    results, errors = [None] * num_requests, []
    start = time.perf_counter()

    def worker(i):
        try:
            results[i] = one_request(url, prompts[i], output_len, timeout)
        except Exception as e:  # noqa: BLE001 - counted, reported
            errors.append(repr(e))
        finally:
            sem.release()

    threads = []
    for i, at in enumerate(arrivals):
        delay = start + at - time.perf_counter()
        if delay > 0:
            time.sleep(delay)
        sem.acquire()
        th = threading.Thread(target=worker, args=(i,), daemon=True)
        th.start()
        threads.append(th)
    for th in threads:
        th.join()
    wall = time.perf_counter() - start
    ok = [r for r in results if r is not None]
    ttft = [r[0] for r in ok if r[0] is not None]
    itl = [g for r in ok for g in r[1]]
    lat = [r[2] for r in ok]
    out_tok = sum(r[3] for r in ok)
    in_tok = sum(len(p) for p, r in zip(prompts, results) if r is not None)
    ms = 1e3
    return {
        "bench": "serving", "requests": num_requests, "completed": len(ok), "errors": len(errors),
        "concurrency": concurrency, "request_rate": None if request_rate == float("inf") else request_rate,
        "wall_s": round(wall, 3), "request_throughput": len(ok) / wall,
        "input_tok_s": in_tok / wall, "output_tok_s": out_tok / wall, "total_tok_s": (in_tok + out_tok) / wall,
        "ttft_ms": {f"p{int(q * 100)}": (_pct(ttft, q) or 0) * ms for q in (0.5, 0.9, 0.99)},
        "itl_ms": {f"p{int(q * 100)}": (_pct(itl, q) or 0) * ms for q in (0.5, 0.9, 0.99)},
        "latency_ms": {f"p{int(q * 100)}": (_pct(lat, q) or 0) * ms for q in (0.5, 0.9, 0.99)},
        "first_error": errors[0] if errors else None,
    }


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--url", default="http://127.0.0.1:8001")
    ap.add_argument("--num-requests", type=int, default=128)
    ap.add_argument("--concurrency", type=int, default=32)
    ap.add_argument("--request-rate", type=float, default=float("inf"), help="requests/s (Poisson); inf = at once")
    ap.add_argument("--input-len", default="512:4096", help="prompt tokens, N or LO:HI (uniform)")
    ap.add_argument("--output-len", type=int, default=128)
    ap.add_argument("--vocab", type=int, default=256, help="token-id range (256: byte tokenizer)")
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    lo, _, hi = args.input_len.partition(":")
    res = run(args.url, args.num_requests, args.concurrency, args.request_rate, (int(lo), int(hi or lo)),
              args.output_len, args.vocab, args.seed)
    print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()
