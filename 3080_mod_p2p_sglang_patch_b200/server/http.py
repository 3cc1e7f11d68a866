"""The HTTP front end over an EngineServer: OpenAI completions and chat,
sglang's /generate and admin endpoints, health and Prometheus metrics."""
import itertools
import json
import threading
import time

from ..engine.tokenizer import ByteTokenizer
from .loop import EngineServer, _find_stop, _held_back, _stop_prefix


def build_app(server: EngineServer, model_name: str, tokenizer=None, api_key: str = None):
    """FastAPI app with /health, /metrics, /v1/models, /v1/completions,
    /v1/chat/completions and /generate (plain or streamed; greedy or
    sampled; stop token ids and stop strings). ``api_key``: requests to the
    model endpoints need ``Authorization: Bearer <api_key>`` (/health,
    /health_generate and /metrics stay open for probes)."""
    import hmac

    from fastapi import FastAPI, HTTPException, Request
    from fastapi.concurrency import iterate_in_threadpool, run_in_threadpool
    from fastapi.responses import JSONResponse, StreamingResponse

    tok = tokenizer or ByteTokenizer()
    app = FastAPI()
    ids = itertools.count()

    if api_key:
        @app.middleware("http")
        async def _auth(request: Request, call_next):
            if request.url.path not in ("/health", "/health_generate", "/metrics"):
                got = request.headers.get("authorization", "")
                if not hmac.compare_digest(got.encode(), f"Bearer {api_key}".encode()):
                    return JSONResponse({"error": {"message": "invalid or missing API key"}}, status_code=401)
            return await call_next(request)

    def _prompt_ids(p):
        if isinstance(p, list) and all(isinstance(i, int) for i in p):
            return p
        if isinstance(p, str):
            return tok.encode(p)
        raise HTTPException(400, "prompt must be a string or a list of token ids")

    def _stop(body):
        """Stop token ids: ``stop_token_ids``, else none with ``ignore_eos``,
        else None (the server's default, the checkpoint's EOS ids)."""
        ids_ = body.get("stop_token_ids")
        if ids_ is None:
            return [] if body.get("ignore_eos") else None
        return [int(t) for t in ids_]

    def _stop_strs(body):
        """OpenAI ``stop``: a string or a list of strings."""
        st = body.get("stop")
        if st is None:
            return ()
        if isinstance(st, str):
            return (st,)
        if isinstance(st, list) and all(isinstance(x, str) for x in st):
            return tuple(st)
        raise HTTPException(400, "stop must be a string or a list of strings")

    def _text(out, stops):
        """Decoded text, ending before the first stop string."""
        text = tok.decode(out)
        i = _find_stop(text, stops) if stops else -1
        return text if i < 0 else text[:i]

    def _sampling(body):
        """The fields of engine.sampling.SamplingParams, in order (temperature,
        top_k, top_p, seed, presence / frequency / repetition penalties,
        logit_bias, min tokens), or None for plain greedy decoding."""
        t = float(body.get("temperature") or 0.0)
        try:
            bias = tuple(sorted((int(k), float(v)) for k, v in (body.get("logit_bias") or {}).items()))
        except (TypeError, ValueError, AttributeError) as e:
            raise HTTPException(400, "logit_bias must map token ids to numbers") from e
        adj = (float(body.get("presence_penalty") or 0.0), float(body.get("frequency_penalty") or 0.0),
               float(body.get("repetition_penalty") or 1.0), bias,
               int(body.get("min_tokens") or body.get("min_new_tokens") or 0))
        if adj[2] <= 0:
            raise HTTPException(400, "repetition_penalty must be positive")
        if t <= 0.0 and adj == (0.0, 0.0, 1.0, (), 0):
            return None
        seed = body.get("seed")
        return (max(t, 0.0), int(body.get("top_k") or 0), float(body.get("top_p") or 1.0),
                None if seed is None else int(seed)) + adj

    def _run(prompt, max_tokens, stop=None, sampling=None, stops=(), logprobs=None, prompt_logprobs=False,
             name=None, timeout=None):
        """(output ids, finish reason, per-token logprobs, prompt logprobs)."""
        try:
            p = server._submit_pending(prompt, max_tokens, timeout=timeout, stop_ids=stop, sampling=sampling,
                                       stop_strs=stops, detok=tok.decode, logprobs=logprobs,
                                       prompt_logprobs=prompt_logprobs, name=name)
            return p.output, p.reason, p.token_logprobs, p.prompt_token_logprobs
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        except (RuntimeError, TimeoutError) as e:
            raise HTTPException(503, str(e)) from e

    def _tok_str(t):
        return tok.decode([t])

    def _completion_logprobs(out, lps):
        """OpenAI completions ``logprobs``: tokens, token_logprobs,
        top_logprobs (token text -> logprob), text_offset. An entry of None
        (the first echoed prompt token) has no logprob."""
        toks = [_tok_str(t) for t in out]
        offs, o = [], 0
        for t in toks:
            offs.append(o)
            o += len(t)
        return {"tokens": toks, "token_logprobs": [None if e is None else e[0] for e in lps],
                "top_logprobs": [None if e is None else {_tok_str(i): v for i, v in e[1]} for e in lps],
                "text_offset": offs}

    def _chat_logprobs(out, lps):
        """OpenAI chat ``logprobs``: content = [{token, logprob, bytes, top_logprobs}]."""
        def item(t, lp):
            s_ = _tok_str(t)
            return {"token": s_, "logprob": lp, "bytes": list(s_.encode("utf-8"))}
        return {"content": [{**item(t, lp), "top_logprobs": [item(i, v) for i, v in top]}
                            for t, (lp, top) in zip(out, lps)]}

    def _n(body):
        n = int(body.get("n") or 1)
        if n < 1 or n > 16:
            raise HTTPException(400, "n must lie in 1..16")
        if n > 1 and body.get("stream"):
            raise HTTPException(400, "n > 1 is not supported with stream")
        return n

    async def _run_n(n, prompt, max_tokens, stop, sampling, stops, lp, plp=False):
        """n independent requests for one prompt (choice i draws with seed + i
        when the request is seeded); each result as ``_run`` returns it."""
        import asyncio

        def samp(i):
            if sampling is None or sampling[3] is None:
                return sampling
            return sampling[:3] + (sampling[3] + i,) + sampling[4:]

        return await asyncio.gather(*[run_in_threadpool(_run, prompt, max_tokens, stop, samp(i), stops, lp, plp)
                                      for i in range(n)])

    def _usage_n(prompt, outs):
        c = sum(len(o) for o in outs)
        return {"prompt_tokens": len(prompt), "completion_tokens": c, "total_tokens": len(prompt) + c}

    def _usage(prompt, out):
        return {"prompt_tokens": len(prompt), "completion_tokens": len(out), "total_tokens": len(prompt) + len(out)}

    def _check(prompt, max_tokens):
        try:
            server._enqueue_check(prompt, max_tokens)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        if server.overloaded():  # before a stream starts: a status code, not an error event
            raise HTTPException(503, "server overloaded")

    def _no_usage(body):
        """OpenAI ``stream_options.include_usage: false``: the last chunk
        carries no usage (by default it does)."""
        so = body.get("stream_options") or {}
        return isinstance(so, dict) and so.get("include_usage") is False

    def _sse(prompt, max_tokens, chunk_of, stop=None, sampling=None, stops=(), lp=None, lp_fmt=None,
             usage=True):
        """Server-sent events: one chunk per engine step's new tokens (the text
        delta of the decoded output, cut before a stop string), a last chunk
        with finish_reason and usage, then [DONE]. A client that disconnects
        closes the generator, which aborts the request. With ``lp`` (k
        alternatives) each chunk carries ``lp_fmt(tokens, logprobs)`` of its
        tokens."""
        def gen():
            out, reason, sent = [], [], ""
            fin = None
            try:
                stream = server.submit_stream(prompt, max_tokens, stop_ids=stop, reason_out=reason,
                                              sampling=sampling, stop_strs=stops, detok=tok.decode, logprobs=lp)
                try:
                    for item in stream:
                        toks, lps = item if lp is not None else (item, None)
                        out += toks
                        hit = bool(stops) and _find_stop(tok.decode(out), stops) >= 0
                        text = _text(out, stops)
                        if stops and not hit:
                            text = text[:len(text) - _held_back(text, stops)]
                        delta, sent = text[len(sent):], text
                        obj = chunk_of(toks, delta, None, None)
                        if lp is not None:
                            obj["choices"][0]["logprobs"] = lp_fmt(toks, lps)
                        yield "data: " + json.dumps(obj) + "\n\n"
                        if hit:
                            fin = "stop"  # the server loop drops the request on every rank
                            break
                finally:
                    stream.close()
                fin = fin or (reason[0] if reason else "length")
                if fin == "stop" and stops:
                    out = out[:_stop_prefix(out, stops, tok.decode) or len(out)]
                rest = _text(out, stops)[len(sent):]  # text held back for a stop string that never came
                yield "data: " + json.dumps(chunk_of([], rest, fin, _usage(prompt, out) if usage else None)) + "\n\n"
            except (RuntimeError, TimeoutError) as e:
                yield "data: " + json.dumps({"error": {"message": str(e)}}) + "\n\n"
            yield "data: [DONE]\n\n"

        return StreamingResponse(iterate_in_threadpool(gen()), media_type="text/event-stream")

    @app.get("/health")
    def health():
        """200 while serving; 503 once the server stopped or the communicator
        holds a device error (a timed-out peer wait), so a load balancer or the
        data-parallel router can see it."""
        tp = getattr(server.engine, "tp", None)
        comm = getattr(tp, "ca_comm", None) if tp is not None else None
        err = comm.err() if comm is not None else 0
        if server._stopped.is_set() or err:
            return JSONResponse({"status": "unhealthy", "communicator_error": err, **server.stats}, status_code=503)
        return {"status": "ok", **server.stats}

    @app.get("/metrics")
    def metrics():
        """Prometheus text format: request / token / step counters, latency
        quantiles, and the communicator's calls per path (one-shot, two-shot,
        NVLS, fused, NCCL fallback, errors) when the engine runs on MailboxAR."""
        from fastapi.responses import PlainTextResponse

        return PlainTextResponse(render_metrics(server), media_type="text/plain; version=0.0.4")

    @app.post("/flush_cache")
    def flush_cache():
        server.flush_cache()
        return {"status": "ok"}

    @app.get("/get_model_info")
    def model_info():
        eng = server.engine
        cfg = getattr(eng, "cfg", None)
        return {"model_path": model_name, "is_generation": True,
                "max_seq": getattr(eng, "max_seq", None), "tp_size": server.world,
                "vocab_size": getattr(cfg, "vocab", None)}

    @app.get("/get_server_info")
    def server_info():
        eng = server.engine
        return {"tp_size": server.world, "max_batch": getattr(eng, "max_batch", None),
                "chunk": getattr(eng, "chunk", None), "impl": getattr(eng, "impl", None),
                "prefix_cache": getattr(eng, "prefix_cache", None) is not None,
                "max_queued_requests": server.max_queued, **server.stats}

    @app.post("/abort_request")
    def abort_request(body: dict):
        """sglang's abort by client request id (the ``rid`` given to
        /generate): the request ends at the next step on every rank and its
        caller gets the tokens so far, with finish reason "abort"."""
        rid = body.get("rid")
        if rid is None:
            raise HTTPException(400, "rid is required")
        return {"rid": rid, "aborted": server.abort_request(rid)}

    @app.get("/health_generate")
    async def health_generate():
        """Health by generating one token from a one-token prompt through
        the whole loop (every rank steps); 503 if that fails or takes more
        than 30 s."""
        try:
            await run_in_threadpool(server._submit_pending, [0], 1, 30.0)
        except (ValueError, RuntimeError, TimeoutError) as e:
            return JSONResponse({"status": "unhealthy", "error": str(e)}, status_code=503)
        return {"status": "ok"}

    @app.post("/tokenize")
    def tokenize(body: dict):
        return {"tokens": tok.encode(str(body.get("text", "")))}

    @app.post("/detokenize")
    def detokenize(body: dict):
        return {"text": tok.decode([int(t) for t in body.get("tokens") or []])}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "mailbox-ar-b200"}]}

    def _prompt_batch(p):
        """OpenAI ``prompt``: a string, a token-id list, or a list of either
        (several prompts in one request)."""
        if isinstance(p, list) and p and all(isinstance(x, (str, list)) for x in p):
            return [_prompt_ids(x) for x in p]
        return [_prompt_ids(p)]

    @app.post("/v1/completions")
    async def completions(body: dict):
        import asyncio

        prompts = _prompt_batch(body.get("prompt", ""))
        prompt = prompts[0]
        max_tokens = int(body.get("max_tokens", 16))
        echo = bool(body.get("echo"))
        score_only = echo and max_tokens == 0  # scoring: the prompt's logprobs, nothing generated
        if score_only:
            max_tokens = 1
        stop, stops = _stop(body), _stop_strs(body)
        lp = body.get("logprobs")
        lp = None if lp is None or lp is False else int(lp)
        if body.get("stream"):
            _n(body)
            if len(prompts) > 1:
                raise HTTPException(400, "several prompts are not supported with stream")
            if echo:
                raise HTTPException(400, "echo is not supported with stream")
            _check(prompt, max_tokens)
            cid, created = f"cmpl-{next(ids)}", int(time.time())
            return _sse(prompt, max_tokens, lambda toks, text, fin, usage: {
                "id": cid, "object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "text": text, "token_ids": toks, "finish_reason": fin, "logprobs": None}],
                **({"usage": usage} if usage else {})}, stop, _sampling(body), stops, lp, _completion_logprobs,
                not _no_usage(body))
        n = _n(body)
        for pr in prompts:  # refuse the whole request before running any of it
            _check(pr, max_tokens)
        per_prompt = await asyncio.gather(*[_run_n(n, pr, max_tokens, stop, _sampling(body), stops, lp,
                                                   echo and lp is not None) for pr in prompts])
        choices, outs = [], []
        for pr, runs in zip(prompts, per_prompt):   # choices: prompt-major, then n
            for out, fin, lps, plps in runs:
                if score_only:
                    out, lps, fin = [], [], "length"
                text = _text(out, stops)
                logprobs = None
                if lp is not None:
                    logprobs = _completion_logprobs((pr if echo else []) + out, (plps if echo else []) + lps)
                if echo:
                    text = tok.decode(pr) + text
                choices.append({"index": len(choices), "text": text, "token_ids": out, "finish_reason": fin,
                                "logprobs": logprobs})
                outs.append(out)
        usage = _usage_n(prompt, outs)
        usage["prompt_tokens"] = sum(len(pr) for pr in prompts) * n
        usage["total_tokens"] = usage["prompt_tokens"] + usage["completion_tokens"]
        return {"id": f"cmpl-{next(ids)}", "object": "text_completion", "created": int(time.time()),
                "model": model_name, "choices": choices, "usage": usage}

    @app.post("/v1/chat/completions")
    async def chat(body: dict):
        msgs = body.get("messages") or []
        prompt = tok.chat(msgs)
        max_tokens = int(body.get("max_completion_tokens") or body.get("max_tokens") or 16)
        stop, stops = _stop(body), _stop_strs(body)
        lp = int(body.get("top_logprobs") or 0) if body.get("logprobs") else None
        if body.get("stream"):
            _n(body)
            _check(prompt, max_tokens)
            cid, created = f"chatcmpl-{next(ids)}", int(time.time())
            return _sse(prompt, max_tokens, lambda toks, text, fin, usage: {
                "id": cid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                "choices": [{"index": 0, "delta": {"content": text} if (toks or text) else {},
                             "token_ids": toks, "finish_reason": fin, "logprobs": None}],
                **({"usage": usage} if usage else {})}, stop, _sampling(body), stops, lp, _chat_logprobs,
                not _no_usage(body))
        runs = await _run_n(_n(body), prompt, max_tokens, stop, _sampling(body), stops, lp)
        choices = [{"index": i, "message": {"role": "assistant", "content": _text(out, stops)}, "token_ids": out,
                    "finish_reason": fin, "logprobs": _chat_logprobs(out, lps) if lp is not None else None}
                   for i, (out, fin, lps, _) in enumerate(runs)]
        return {"id": f"chatcmpl-{next(ids)}", "object": "chat.completion", "created": int(time.time()),
                "model": model_name, "choices": choices, "usage": _usage_n(prompt, [r[0] for r in runs])}

    @app.post("/generate")
    async def generate(body: dict):
        """sglang's native API: ``text`` (or ``input_ids``) and a
        ``sampling_params`` dict (max_new_tokens, temperature, top_k, top_p,
        seed, stop, stop_token_ids). Returns ``text``, ``output_ids`` and
        ``meta_info`` (prompt / completion tokens, finish_reason); with
        ``stream`` the same objects, cumulative, as server-sent events. A
        batch (``text`` a list of strings, or ``input_ids`` a list of id
        lists; ``sampling_params`` and ``rid`` one per item or shared) returns
        a list, one result per item, in order."""
        key = "input_ids" if body.get("input_ids") is not None else "text"
        src = body.get(key, "")
        if isinstance(src, list) and src and all(isinstance(x, (str, list)) for x in src):
            return await _generate_batch(body, key, src)
        if body.get("input_ids") is not None:
            prompt = _prompt_ids(body["input_ids"])
        else:
            prompt = _prompt_ids(body.get("text", ""))
        sp = dict(body.get("sampling_params") or {})
        max_new = int(sp.get("max_new_tokens", 128))
        stop, stops = _stop(sp), _stop_strs(sp)
        sampling = _sampling(sp)
        want_lp = bool(body.get("return_logprob"))
        top_n = int(body.get("top_logprobs_num") or 0)
        start = body.get("logprob_start_len")
        score_prompt = want_lp and start is not None and int(start) >= 0
        rid = body.get("rid")
        if rid is not None and not isinstance(rid, (str, int)):
            raise HTTPException(400, "rid must be a string (one request per call)")

        def _lp_list(toks, lps):
            """sglang's [logprob, token id, None] triples (and top-n lists)."""
            vals = [[None if e is None else e[0], t, None] for t, e in zip(toks, lps)]
            tops = [None if e is None else [[v, i, None] for i, v in e[1]] for e in lps]
            return vals, tops

        def result(out, fin, lps=(), plps=()):
            meta = {"prompt_tokens": len(prompt), "completion_tokens": len(out), "finish_reason": {"type": fin}}
            if want_lp:
                meta["output_token_logprobs"], tops = _lp_list(out, lps)
                if top_n:
                    meta["output_top_logprobs"] = tops
                if score_prompt:
                    k = int(start)
                    meta["input_token_logprobs"], itops = _lp_list(prompt[k:], list(plps)[k:])
                    if top_n:
                        meta["input_top_logprobs"] = itops
            if rid is not None:
                meta["id"] = rid
            return {"text": _text(out, stops), "output_ids": out, "meta_info": meta}

        if body.get("stream"):
            if score_prompt:
                raise HTTPException(400, "logprob_start_len is not supported with stream")
            _check(prompt, max_new)
            lpk = top_n if want_lp else None

            def gen():
                out, reason, lps = [], [], []
                try:
                    stream = server.submit_stream(prompt, max_new, stop_ids=stop, reason_out=reason,
                                                  sampling=sampling, stop_strs=stops, detok=tok.decode, name=rid,
                                                  logprobs=lpk)
                    fin = None
                    try:
                        for item in stream:
                            toks, new = item if lpk is not None else (item, [])
                            out += toks
                            lps += new
                            if stops and _find_stop(tok.decode(out), stops) >= 0:
                                fin = "stop"
                                break
                            yield "data: " + json.dumps(result(out, None, lps)) + "\n\n"
                    finally:
                        stream.close()
                    fin = fin or (reason[0] if reason else "length")
                    if fin == "stop" and stops:
                        out = out[:_stop_prefix(out, stops, tok.decode) or len(out)]
                    yield "data: " + json.dumps(result(out, fin, lps[:len(out)])) + "\n\n"
                except (ValueError, RuntimeError, TimeoutError) as e:
                    yield "data: " + json.dumps({"error": {"message": str(e)}}) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(iterate_in_threadpool(gen()), media_type="text/event-stream")
        out, fin, lps, plps = await run_in_threadpool(_run, prompt, max_new, stop, sampling, stops,
                                                      top_n if want_lp else None, score_prompt, rid)
        return result(out, fin, lps, plps)

    async def _generate_batch(body, key, items):
        import asyncio

        if body.get("stream"):
            raise HTTPException(400, "a batch is not supported with stream")
        n = len(items)

        def per_item(field, default):
            v = body.get(field, default)
            if isinstance(v, list):
                if len(v) != n:
                    raise HTTPException(400, f"{field} has {len(v)} entries for {n} prompts")
                return v
            return [v] * n

        sps, rids = per_item("sampling_params", {}), per_item("rid", None)
        if rids[0] is not None and len(set(rids)) != n:
            raise HTTPException(400, "rid values must differ within a batch")
        for x, sp in zip(items, sps):  # refuse the whole batch before running any of it
            _check(_prompt_ids(x), int((sp or {}).get("max_new_tokens", 128)))
        subs = [{**body, key: x, "sampling_params": sp, "rid": r} for x, sp, r in zip(items, sps, rids)]
        return list(await asyncio.gather(*[generate(sb) for sb in subs]))

    return app


def _quantiles(xs, qs=(0.5, 0.9, 0.99)):
    v = sorted(xs)
    return {q: v[min(len(v) - 1, int(q * len(v)))] for q in qs} if v else {}


def render_metrics(server: "EngineServer") -> str:
    """The server's metrics in Prometheus text exposition format."""
    lines = []

    def metric(name, kind, help_, samples):
        lines.append(f"# HELP {name} {help_}")
        lines.append(f"# TYPE {name} {kind}")
        for labels, value in samples:
            lab = "{" + ",".join(f'{k}="{v}"' for k, v in labels.items()) + "}" if labels else ""
            lines.append(f"{name}{lab} {value}")

    st = server.stats
    metric("mbx_requests_total", "counter", "Requests admitted.", [({}, st["requests"])])
    metric("mbx_prompt_tokens_total", "counter", "Prompt tokens admitted.", [({}, st["prompt_tokens"])])
    metric("mbx_generation_tokens_total", "counter", "Tokens generated by finished requests.",
           [({}, st["completion_tokens"])])
    metric("mbx_engine_steps_total", "counter", "Engine steps (prefill chunks and decode batches).",
           [({}, st["steps"])])
    for name, xs, help_ in (("mbx_time_to_first_token_seconds", server.ttft, "Time to first token."),
                            ("mbx_inter_token_latency_seconds", server.itl, "Gap between generated tokens.")):
        metric(name, "summary", help_, [({"quantile": q}, v) for q, v in _quantiles(xs).items()] +
               [({"stat": "count"}, len(xs))])
    eng = server.engine
    tp = getattr(eng, "tp", None)
    comm = getattr(tp, "ca_comm", None) if tp is not None else None
    if comm is not None:
        metric("mbx_allreduce_calls_total", "counter", "In-house collective calls by path.",
               [({"path": k}, v) for k, v in sorted(comm.counters.items())])
        metric("mbx_communicator_error", "gauge", "Sticky device error code (0 = ok).", [({}, comm.err())])
    metric("mbx_requests_in_flight", "gauge", "Requests submitted and not finished.", [({}, server._live)])
    sched = getattr(eng, "sched", None)
    if sched is not None:
        for name, attr, help_ in (("mbx_num_queue_reqs", "waiting", "Requests waiting for admission."),
                                  ("mbx_num_prefill_reqs", "prefilling", "Requests with prompt tokens left."),
                                  ("mbx_num_running_reqs", "running", "Requests decoding.")):
            if hasattr(sched, attr):
                metric(name, "gauge", help_, [({}, len(getattr(sched, attr)))])
    alloc = getattr(getattr(eng, "kv", None), "alloc", None)
    if alloc is not None and alloc.capacity:
        metric("mbx_kv_cache_usage", "gauge", "Fraction of KV cache pages in use (prefix-cache pages included).",
               [({}, round((alloc.capacity - alloc.free) / alloc.capacity, 6))])
    pc = getattr(eng, "prefix_cache", None)
    if pc is not None:
        metric("mbx_prefix_cache_hit_pages_total", "counter", "KV pages served from the prefix cache.",
               [({}, pc.hits)])
    return "\n".join(lines) + "\n"


def start_http(app, host: str, port: int):
    """Run uvicorn in a daemon thread; returns (server, thread)."""
    import uvicorn

    config = uvicorn.Config(app, host=host, port=port, log_level="warning", lifespan="off")
    srv = uvicorn.Server(config)
    th = threading.Thread(target=srv.run, daemon=True, name="http")
    th.start()
    deadline = time.time() + 30
    while not srv.started and th.is_alive() and time.time() < deadline:
        time.sleep(0.02)
    if not srv.started:
        raise RuntimeError(f"HTTP server did not start on {host}:{port}")
    return srv, th
