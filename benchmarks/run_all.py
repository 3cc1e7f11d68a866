"""Run the benchmark set at one GPU count and collect every JSON result line
into one file (the numbers behind the results tables).

    python benchmarks/run_all.py --gpus 8 --out results_tp8.jsonl
    python benchmarks/run_all.py --gpus 2 --only bench,allreduce --dry-run

Each benchmark runs as its own process: ``python`` for one GPU,
``torch.distributed.run`` on 127.0.0.1 otherwise, under a time limit. Lines
of its output that parse as JSON objects are appended to ``--out`` with the
benchmark's name and command; a failed or timed-out benchmark is recorded
with its exit code and the end of its output, and the rest still run.
"""
import argparse
import json
import os
import socket
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# name -> (script, extra arguments, minimum GPUs)
BENCHES = {
    "bench": ("bench.py", ["--steps", "3", "--warmup", "3"], 1),
    "bench_torch": ("bench.py", ["--steps", "3", "--warmup", "3", "--impl", "torch"], 1),
    "decode": ("benchmarks/decode_bench.py", [], 1),
    "decode_torch": ("benchmarks/decode_bench.py", ["--impl", "torch"], 1),
    "decode_int4": ("benchmarks/decode_bench.py", ["--int4"], 1),
    "perplexity": ("benchmarks/perplexity.py", ["--model", "tiny", "--compare", "oracle"], 1),
    "allreduce": ("benchmarks/allreduce_sweep.py", ["--graph"], 2),
    "fused_ar": ("benchmarks/fused_ar_bench.py", [], 2),
    "push": ("benchmarks/push_bench.py", [], 2),
    "serve_70b": ("benchmarks/serve_bench.py", ["--model", "70b"], 8),
}


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def command(name: str, gpus: int):
    script, extra, _ = BENCHES[name]
    path = os.path.join(ROOT, script)
    gpu_args = ["--gpus", str(gpus)] if script == "bench.py" else []
    if gpus == 1:
        return [sys.executable, path, *gpu_args, *extra]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr=127.0.0.1", f"--master-port={_port()}", path, *gpu_args, *extra]


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--only", default=None, help=f"comma-separated subset of: {', '.join(BENCHES)}")
    ap.add_argument("--out", default="results.jsonl")
    ap.add_argument("--timeout", type=float, default=1800.0, help="seconds per benchmark")
    ap.add_argument("--dry-run", action="store_true", help="print the commands only")
    args = ap.parse_args(argv)
    names = args.only.split(",") if args.only else list(BENCHES)
    unknown = [n for n in names if n not in BENCHES]
    if unknown:
        raise SystemExit(f"unknown benchmarks: {', '.join(unknown)}")
    runs = [(n, command(n, args.gpus)) for n in names if BENCHES[n][2] <= args.gpus]
    if args.dry_run:
        for n, cmd in runs:
            print(n, " ".join(cmd))
        return runs
    env = dict(os.environ)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    with open(args.out, "a") as out:
        for n, cmd in runs:
            t0 = time.time()
            try:
                p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=args.timeout)
                code, text = p.returncode, p.stdout + p.stderr
            except subprocess.TimeoutExpired as e:
                code, text = "timeout", (e.stdout or b"").decode(errors="replace") if isinstance(e.stdout, bytes) \
                    else (e.stdout or "")
            found = 0
            for line in text.splitlines():
                line = line.strip()
                if line.startswith("{") and line.endswith("}"):
                    try:
                        rec = json.loads(line)
                    except ValueError:
                        continue
                    out.write(json.dumps({"bench": n, "gpus": args.gpus, "cmd": " ".join(cmd[1:]), **rec}) + "\n")
                    found += 1
            if code != 0:
                out.write(json.dumps({"bench": n, "gpus": args.gpus, "cmd": " ".join(cmd[1:]), "exit": code,
                                      "tail": text[-2000:]}) + "\n")
            out.flush()
            print(f"{n}: exit {code}, {found} result lines, {time.time() - t0:.0f} s", flush=True)
    return runs


if __name__ == "__main__":
    main()
