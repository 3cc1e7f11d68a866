"""Command line of the server: sglang-style flags, the --tp / --dp
launchers, and ``main`` (one process per GPU)."""
import argparse
import dataclasses
import datetime
import logging
import os
import signal
import subprocess
import sys

from ..engine.tokenizer import ByteTokenizer, HFTokenizer, load_chat_template
from .http import build_app, start_http
from .loop import EngineServer

logger = logging.getLogger(__name__)


RANDOM_MODELS = ("8b", "70b", "tiny")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="OpenAI-compatible TP serving on B200 (MailboxAR collectives).")
    ap.add_argument("--model", default="8b",
                    help="a Hugging Face checkpoint directory, or 8b | 70b | tiny (random weights)")
    ap.add_argument("--model-path", default=None, help="Hugging Face checkpoint directory (safetensors)")
    ap.add_argument("--tp", "--tp-size", dest="tp", type=int, default=None,
                    help="tensor-parallel ranks (one GPU each); started here unless launched by torchrun")
    ap.add_argument("--dp", "--dp-size", dest="dp", type=int, default=1,
                    help="data-parallel replicas, each a TP group on its own GPUs, behind one router")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8001)
    ap.add_argument("--api-key", default=None, help="require Authorization: Bearer <key> on the model endpoints")
    ap.add_argument("--served-model-name", default=None, help="model id reported by /v1/models")
    ap.add_argument("--log-requests", action="store_true", help="one JSON log line per finished request")
    ap.add_argument("--max-queued-requests", type=int, default=None,
                    help="refuse new requests (HTTP 503) while this many are queued or running")
    # sglang launch flags with the same meaning here
    ap.add_argument("--dtype", default="auto", choices=["auto", "bfloat16", "bf16"],
                    help="compute dtype: bf16 (auto)")
    ap.add_argument("--kv-cache-dtype", default="auto", choices=["auto", "bfloat16", "bf16"],
                    help="KV cache dtype: bf16 (auto)")
    ap.add_argument("--quantization", default=None, choices=["awq", "awq_marlin"],
                    help="AWQ checkpoints: keep the int4 weights packed (same as --int4-weights)")
    ap.add_argument("--random-seed", "--seed", dest="seed", type=int, default=0,
                    help="random weights and unseeded sampling draws")
    ap.add_argument("--log-level", default="info", choices=["debug", "info", "warning", "error"])
    ap.add_argument("--max-total-tokens", type=int, default=None, help="KV cache capacity in tokens")
    ap.add_argument("--cuda-graph-bs", type=int, nargs="+", default=None,
                    help="decode batch sizes captured as CUDA graphs (default 1 8 32 64)")
    ap.add_argument("--cuda-graph-max-bs", type=int, default=None,
                    help="largest decode batch captured as a CUDA graph")
    ap.add_argument("--disable-radix-cache", action="store_true",
                    help="no prefix sharing (the default unless --prefix-cache)")
    ap.add_argument("--disable-custom-all-reduce", action="store_true",
                    help="TP allreduces on NCCL even with SGLANG_MAILBOX_AR=1 (sglang's switch for its custom "
                         "allreduce, the slot MailboxAR fills)")
    ap.add_argument("--trust-remote-code", action="store_true",
                    help="accepted for sglang command lines; no checkpoint code is ever run")
    ap.add_argument("--tokenizer-path", default=None,
                    help="tokenizer directory (default: the checkpoint's own; with random weights, "
                         "replaces the byte tokenizer)")
    ap.add_argument("--chat-template", default=None,
                    help="Jinja chat template (a file, or the template text) instead of the checkpoint's own")
    ap.add_argument("--max-batch", "--max-running-requests", dest="max_batch", type=int, default=64)
    ap.add_argument("--max-seq", "--context-length", dest="max_seq", type=int, default=None,
                    help="longest prompt + generation (default: the model's positions, at most 16384 with "
                         "random weights, 8192 with a checkpoint)")
    ap.add_argument("--chunk", "--chunked-prefill-size", dest="chunk", type=int, default=1024)
    ap.add_argument("--impl", default="native", choices=["native", "torch", "oracle"],
                    help="native: the sm_100a kernels; torch: cuBLAS + NCCL baseline; oracle: fp32 PyTorch "
                         "restatement (with --device cpu: no GPU, for API development and tests)")
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"],
                    help="cpu needs --impl oracle; ranks then talk over gloo")
    ap.add_argument("--no-graphs", "--disable-cuda-graph", dest="no_graphs", action="store_true")
    ap.add_argument("--prefix-cache", action="store_true", help="share the KV pages of common prompt prefixes")
    ap.add_argument("--schedule-policy", default=None, choices=["fcfs", "lpm"],
                    help="admission order: arrival (fcfs) or longest cached prefix first (lpm; the default with "
                         "--prefix-cache)")
    ap.add_argument("--graph-sampled-decode", action="store_true",
                    help="decode batches that sample (or need logprobs / logit adjustments) replay a CUDA graph "
                         "ending in the full logits instead of running eagerly")
    ap.add_argument("--enable-mixed-chunk", dest="mixed_chunk", action="store_true",
                    help="prefill batches also carry the running requests' decode tokens")
    ap.add_argument("--int4-weights", action="store_true",
                    help="keep an AWQ checkpoint's linears packed as int4 (int4 GEMV for decode) instead of "
                         "expanding them to bf16 at load")
    ap.add_argument("--mem-fraction-static", dest="mem_fraction", type=float, default=None,
                    help="size the KV cache so weights + cache use this fraction of GPU memory "
                         "(default: room for max-batch requests of max-seq tokens)")
    return ap


def resolve_model(args):
    """(random-weights name or None, checkpoint directory or None) from
    ``--model`` / ``--model-path``: ``--model`` names a directory or one of
    the random-weight configs."""
    if args.model_path:
        return None, args.model_path
    if os.path.isdir(args.model):
        return None, args.model
    if args.model in RANDOM_MODELS:
        return args.model, None
    raise SystemExit(f"--model {args.model!r}: not a directory and not one of {', '.join(RANDOM_MODELS)}")


def _strip_options(argv, names):
    """``argv`` without the options in ``names`` (``--x v`` and ``--x=v``)."""
    rest, skip = [], False
    for a in argv:
        if skip:
            skip = False
        elif a in names:
            skip = True
        elif not a.startswith(tuple(n + "=" for n in names)):
            rest.append(a)
    return rest


def relaunch_command(argv, tp: int, port: int):
    """The torch.distributed.run command that starts ``tp`` ranks of this
    server with ``argv`` minus its ``--tp`` / ``--tp-size`` option."""
    rest = _strip_options(argv, ("--tp", "--tp-size"))
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
            "--master-addr=127.0.0.1", f"--master-port={port}", "-m", f"{_package()}.server", *rest]


def replica_commands(argv, tp: int, dp: int, port: int, visible=None):
    """(environment overrides, command) of each data-parallel replica:
    replica i serves on 127.0.0.1:port + 1 + i over GPUs [i*tp, (i+1)*tp) of
    ``visible`` (the devices this process may use)."""
    gpus = list(visible) if visible is not None else [str(g) for g in range(tp * dp)]
    if len(gpus) < tp * dp:
        raise SystemExit(f"--dp {dp} x --tp {tp} needs {tp * dp} GPUs, {len(gpus)} visible")
    rest = _strip_options(argv, ("--dp", "--dp-size", "--port", "--host", "--tp", "--tp-size"))
    out = []
    for i in range(dp):
        env = {"CUDA_VISIBLE_DEVICES": ",".join(gpus[i * tp:(i + 1) * tp])}
        args_i = rest + ["--host", "127.0.0.1", "--port", str(port + 1 + i)]
        if tp > 1:
            cmd = relaunch_command(args_i, tp, _free_port())
        else:
            cmd = [sys.executable, "-m", f"{_package()}.server", *args_i]
        out.append((env, cmd))
    return out


def _package() -> str:
    """The package root (this module is <root>.server.cli)."""
    return (__package__ or __name__.rsplit(".", 1)[0]).rsplit(".", 1)[0]


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(cmd) -> int:
    """Run the per-rank launcher in the foreground; SIGTERM / SIGINT to this
    process reach it (rank 0 then stops every rank at the same step)."""
    proc = subprocess.Popen(cmd)
    for sig in (signal.SIGINT, signal.SIGTERM):
        signal.signal(sig, lambda signum, _: proc.send_signal(signum))
    return proc.wait()


def _run_replicas(argv, args) -> int:
    """``--dp N``: N replicas (each its own TP group and GPUs) plus the
    data-parallel router on --host:--port in this process."""
    from ..router import Router, build_router_app

    tp = args.tp or 1
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    visible = [v for v in vis.split(",") if v] if vis else None
    if args.device == "cpu":  # no GPUs to partition
        visible = [""] * (tp * args.dp)
    elif visible is None:
        import torch

        visible = [str(g) for g in range(torch.cuda.device_count())]
    procs = []
    for env, cmd in replica_commands(argv, tp, args.dp, args.port, visible):
        procs.append(subprocess.Popen(cmd, env={**os.environ, **env}))
    for sig in (signal.SIGINT, signal.SIGTERM):
        signal.signal(sig, lambda signum, _: [p.send_signal(signum) for p in procs])
    router = Router([f"http://127.0.0.1:{args.port + 1 + i}" for i in range(args.dp)])
    http, _ = start_http(build_router_app(router), args.host, args.port)
    logger.info("data-parallel router at http://%s:%d over %d replicas of TP=%d", args.host, args.port, args.dp, tp)
    codes = [p.wait() for p in procs]
    http.should_exit = True
    return max(codes, key=abs)


def main(argv=None):
    import importlib

    argv = list(sys.argv[1:] if argv is None else argv)
    args = build_parser().parse_args(argv)
    name, model_path = resolve_model(args)
    in_torchrun = "WORLD_SIZE" in os.environ
    if args.tp is not None and args.tp < 1:
        raise SystemExit("--tp must be >= 1")
    if in_torchrun and args.tp is not None and args.tp != int(os.environ["WORLD_SIZE"]):
        raise SystemExit(f"--tp {args.tp} but torchrun started {os.environ['WORLD_SIZE']} ranks")
    if args.dp < 1:
        raise SystemExit("--dp must be >= 1")
    if args.dp > 1:
        if in_torchrun:
            raise SystemExit("--dp starts its own replicas: launch it without torchrun")
        logging.basicConfig(level=logging.INFO, format="%(asctime)s %(name)s %(message)s")
        raise SystemExit(_run_replicas(argv, args))
    if not in_torchrun and (args.tp or 1) > 1:
        raise SystemExit(_run_ranks(relaunch_command(argv, args.tp, _free_port())))

    import torch
    import torch.distributed as dist

    pkg = _package()
    par = importlib.import_module(f"{pkg}.parallel")
    models = importlib.import_module(f"{pkg}.models")
    eng_mod = importlib.import_module(f"{pkg}.engine")
    on_cpu = args.device == "cpu"
    if on_cpu and args.impl != "oracle":
        raise SystemExit("--device cpu runs the oracle model only (--impl oracle)")
    if not on_cpu and not torch.cuda.is_available():
        raise SystemExit("the server needs a CUDA GPU per rank (none visible)")
    logging.basicConfig(level=getattr(logging, args.log_level.upper()), format="%(asctime)s %(name)s %(message)s")
    if args.quantization in ("awq", "awq_marlin"):
        args.int4_weights = True
    if args.disable_radix_cache:
        args.prefix_cache = False
    rank, world, local = par.init_distributed(backend="gloo" if on_cpu else None, timeout_s=600)
    dev = torch.device("cpu") if on_cpu else torch.device("cuda", local)
    # None: follow SGLANG_MAILBOX_AR, like the reference's launch flow (the
    # oracle takes plain torch.distributed collectives)
    no_custom = args.impl == "oracle" or args.disable_custom_all_reduce
    tp = par.TPGroup(None, dev, use_mailbox=False if no_custom else None) if world > 1 else None
    ctrl = dist.new_group(backend="gloo", timeout=datetime.timedelta(days=7)) if world > 1 else None
    opts = dict(max_batch=args.max_batch, chunk=args.chunk, use_graphs=not args.no_graphs,
                impl=args.impl, prefill_graph=(args.impl == "native" and not args.no_graphs),
                prefix_cache=args.prefix_cache, mem_fraction=args.mem_fraction, mixed_chunk=args.mixed_chunk,
                schedule_policy=args.schedule_policy or ("lpm" if args.prefix_cache else "fcfs"),
                sample_in_graphs=args.graph_sampled_decode)
    if args.max_seq is not None:
        opts["max_seq"] = args.max_seq
    if args.max_total_tokens:
        opts["kv_blocks"] = -(-args.max_total_tokens // 16) + 1  # pages of 16 tokens + the reserved page
    opts["seed"] = args.seed
    sizes = tuple(args.cuda_graph_bs) if args.cuda_graph_bs else (1, 8, 32, 64)
    if args.cuda_graph_max_bs:
        sizes = tuple(sorted({x for x in sizes if x <= args.cuda_graph_max_bs} | {args.cuda_graph_max_bs}))
    opts["graph_sizes"] = sizes
    tokenizer = None
    if model_path:
        eng = eng_mod.LLMEngine.from_pretrained(model_path, tp=tp, device=dev, int4_weights=args.int4_weights,
                                                tokenizer_path=args.tokenizer_path, **opts)
        cfg = eng.cfg
        tokenizer = eng.tokenizer
        if tokenizer is None:  # token-id prompts still work
            logger.warning("no tokenizer in %s; using the byte tokenizer", model_path)
        elif args.chat_template:
            tokenizer.tok.chat_template = load_chat_template(args.chat_template)
    else:
        cfg = models.LlamaConfig.by_name(name)
        if args.max_seq is not None and args.max_seq > cfg.max_pos:
            # random weights have no trained position range: a longer context
            # only needs a longer RoPE table (long-prompt prefill benchmarks)
            cfg = dataclasses.replace(cfg, max_pos=args.max_seq)
        opts.setdefault("max_seq", min(16384, cfg.max_pos))
        eng = eng_mod.LLMEngine(cfg, tp=tp, device=dev, **opts)
        if args.tokenizer_path:
            tokenizer = eng.tokenizer = HFTokenizer(args.tokenizer_path, load_chat_template(args.chat_template)
                                                    if args.chat_template else None)
    stop = eng.default_stop_ids
    server = EngineServer(eng, ctrl, rank, world, max_prompt=eng.max_seq, stop_ids=stop,
                          log_requests=args.log_requests, max_queued=args.max_queued_requests)
    http = None
    if rank == 0:
        # Ctrl-C / SIGTERM on rank 0: every rank leaves the loop at the same step
        for sig in (signal.SIGINT, signal.SIGTERM):
            signal.signal(sig, lambda *_: server.stop())
        if tokenizer is None:
            tokenizer = ByteTokenizer(load_chat_template(args.chat_template) if args.chat_template else None)
        http, _ = start_http(build_app(server, args.served_model_name or cfg.name, tokenizer, api_key=args.api_key),
                             args.host, args.port)
        logger.info("serving %s at http://%s:%d (TP=%d, allreduce=%s)", cfg.name, args.host, args.port, world,
                    "MailboxAR" if (tp is not None and tp.ca_comm is not None) else "NCCL")
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        if http is not None:
            http.should_exit = True
        if eng.graphs is not None:
            eng.graphs.close()
        if tp is not None:
            tp.close()
        if world > 1:
            dist.destroy_process_group()
