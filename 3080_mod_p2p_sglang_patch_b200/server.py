"""OpenAI-compatible HTTP front end for the TP engine (the role of sglang's
``launch_server`` in the reference's flow: ``SGLANG_MAILBOX_AR=1 ...
launch_server --tp 2``, reference scripts/sglang-p2p.sh:162; its
prompt-processing bench posts to ``/v1/chat/completions`` and reads
``usage.prompt_tokens``, tests/pp_bench.py:21-29).

    SGLANG_MAILBOX_AR=1 python -m 3080_mod_p2p_sglang_patch_b200.server --model /path/to/ckpt --tp 2
    torchrun --nproc-per-node N -m 3080_mod_p2p_sglang_patch_b200.server --model 8b --port 8001

One process per GPU. ``--tp N`` outside torchrun starts the N ranks itself
(torch.distributed.run on 127.0.0.1); under torchrun the ranks are
torchrun's. sglang's spellings of the common flags are accepted
(``--tp-size``, ``--chunked-prefill-size``, ``--context-length``,
``--max-running-requests``, ``--disable-cuda-graph``).

Rank 0 serves HTTP and owns the request queue; every rank runs the same
engine loop in lockstep: at each iteration rank 0 broadcasts the newly
arrived requests over a gloo control group, every rank adds them in the same
order and runs one engine step (the TP collectives of that step then line up
across ranks). With ``SGLANG_MAILBOX_AR=1`` the TP allreduces go through
MailboxAR, otherwise NCCL.

``--model DIR`` (or ``--model-path DIR``) serves a Hugging Face checkpoint
(safetensors, each rank reads its shards) with the directory's tokenizer
(through transformers, local files only) and its chat template. ``--model
8b|70b|tiny`` runs random weights, and text goes through a byte tokenizer:
UTF-8 bytes are token ids 0..255, generated ids >= 256 decode to nothing.
Token-id prompts (``"prompt": [ids]``) are accepted either way. Decoding is
greedy unless a request sets ``temperature`` (with ``top_p``, ``top_k``,
``seed``).
"""
import argparse
import collections
import datetime
import itertools
import json
import logging
import os
import queue
import signal
import subprocess
import sys
import threading
import time

from .engine.tokenizer import ByteTokenizer, HFTokenizer, load_chat_template  # noqa: F401 - re-exported

logger = logging.getLogger(__name__)


class Overloaded(RuntimeError):
    """The server holds its maximum of queued and running requests."""


class _Pending:
    __slots__ = ("prompt", "max_new", "stop_ids", "sampling", "event", "output", "error", "stream", "req", "sent",
                 "reason", "sid", "stop_strs", "detok", "checked", "stop_hit", "abort_sent", "logprobs",
                 "token_logprobs", "prompt_logprobs", "prompt_token_logprobs", "on_finish")

    def __init__(self, prompt, max_new, stream=False, stop_ids=(), sampling=None, sid=-1, stop_strs=(), detok=None,
                 logprobs=None, prompt_logprobs=False):
        self.prompt = prompt
        self.max_new = max_new
        self.stop_ids = tuple(stop_ids)
        self.sampling = sampling  # (temperature, top_k, top_p, seed) or None
        self.sid = sid            # server-wide request id: the same on every rank
        # stop strings (rank 0): checked on the decoded output after each step
        self.stop_strs = tuple(stop_strs)
        self.detok = detok        # token ids -> text
        self.checked = 0          # output tokens already checked for stop strings
        self.stop_hit = False
        self.abort_sent = False
        self.logprobs = logprobs        # None, or k: per-token logprob + k alternatives
        self.token_logprobs = []
        self.prompt_logprobs = bool(prompt_logprobs)  # also score the prompt (echo)
        self.prompt_token_logprobs = []
        self.on_finish = None     # rank 0: releases the request's place in the overload count
        self.reason = "length"
        self.event = threading.Event()
        self.output = None
        self.error = None
        # streaming: new token ids are put here as they are generated, then None
        self.stream = queue.Queue() if stream else None
        self.req = None  # the engine request (rank 0)
        self.sent = 0    # tokens already streamed

    def finish(self, output=None, error=None):
        if self.on_finish is not None:
            self.on_finish()
            self.on_finish = None
        self.output, self.error = output, error
        if self.stream is not None:
            self.stream.put(None)
        self.event.set()


class EngineServer:
    """Lockstep request loop over the TP ranks.

    ``engine`` needs ``add_request(prompt, max_new) -> request`` (with ``.rid``
    and ``.output``), ``step()``, and ``sched`` with ``has_work()`` and a
    ``finished`` list (``engine.LLMEngine`` has them). ``group`` is a gloo
    process group spanning the TP ranks (None on one rank).
    """

    SHUTDOWN = "__shutdown__"
    FLUSH = "__flush_cache__"

    def __init__(self, engine, group=None, rank: int = 0, world: int = 1, max_prompt: int = None, stop_ids=(),
                 log_requests: bool = False, max_queued: int = None):
        self.engine = engine
        # overload: new requests are refused (HTTP 503) while this many are
        # queued or running; None = no bound
        self.max_queued = max_queued
        self._live = 0                   # submitted and not finished (rank 0)
        self._live_lock = threading.Lock()
        # rank 0 logs one JSON line per finished request (id, tokens, reason, latencies)
        self.log_requests = log_requests
        self.stop_ids = tuple(stop_ids)  # default stop tokens (e.g. the checkpoint's EOS)
        self.group = group
        self.rank = rank
        self.world = world
        self.max_prompt = max_prompt
        self.q = queue.Queue()
        self._by_rid = {}
        self._sids = itertools.count()   # rank 0 numbers requests; the id travels with them
        self._rid_of_sid = {}            # live requests, every rank
        self.stats = {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0, "steps": 0,
                      "control_shm": 0, "control_gloo": 0}  # control-plane exchanges by channel
        # latency samples of finished requests (seconds): time to first token, inter-token gaps
        self.ttft = collections.deque(maxlen=4096)
        self.itl = collections.deque(maxlen=65536)
        self._stopped = threading.Event()
        # Busy steps share the count of new commands over a shared-memory
        # channel (the communicator's CPU transport, ~20 us) instead of a gloo
        # object broadcast (~1 ms) every step; payloads and idle waits still
        # use gloo. Collective: every rank builds its server in the same order.
        self._fast = None
        if group is not None and world > 1:
            self._fast = self._control_channel(group)

    @staticmethod
    def _control_channel(group):
        try:
            import torch

            from .config import CommConfig
            from .parallel.communicator import MailboxAR

            ar = MailboxAR(group, "cpu", config=CommConfig(cpu_slot_bytes=4096))
        except Exception as e:  # noqa: BLE001 - no CPU extension: gloo every step
            logger.warning("control channel unavailable (%s); using gloo every step", e)
            return None
        # MailboxAR agrees on success across ranks, so every rank takes the same path
        return None if ar.disabled else (ar, torch.zeros(4, dtype=torch.float32))

    # ------------------------------------------------------------ rank 0 API
    ABORT = "__abort__"

    def submit(self, prompt: list, max_new: int, timeout: float = None, stop_ids=None, with_reason=False,
               sampling=None, stop_strs=(), detok=None):
        """Called from HTTP threads on rank 0: blocks until the request is done
        and returns the generated token ids (and the finish reason, "length",
        "stop" or "abort", with ``with_reason``). ``stop_ids`` None = the server
        default. ``stop_strs``: generation also ends once ``detok(tokens)``
        contains one of them; the tokens are then cut to the shortest prefix
        whose text contains it."""
        p = self._submit_pending(prompt, max_new, timeout, stop_ids, sampling, stop_strs, detok)
        return (p.output, p.reason) if with_reason else p.output

    def _submit_pending(self, prompt, max_new, timeout=None, stop_ids=None, sampling=None, stop_strs=(), detok=None,
                        logprobs=None, prompt_logprobs=False):
        """``submit`` returning the finished request record (output, reason,
        token_logprobs, prompt_token_logprobs)."""
        p = self._enqueue(prompt, max_new, stream=False, stop_ids=stop_ids, sampling=sampling, stop_strs=stop_strs,
                          detok=detok, logprobs=logprobs, prompt_logprobs=prompt_logprobs)
        if not p.event.wait(timeout):
            raise TimeoutError("request timed out")
        if isinstance(p.error, ValueError):  # the engine rejected the request itself
            raise p.error
        if p.error is not None:
            raise RuntimeError(p.error)
        return p

    def submit_stream(self, prompt: list, max_new: int, timeout: float = None, stop_ids=None, reason_out=None,
                      sampling=None, stop_strs=(), detok=None):
        """Like ``submit`` but yields lists of new token ids as the engine
        produces them (rank 0, from an HTTP thread); the finish reason is
        appended to ``reason_out`` (a list) at the end. Closing the generator
        early (a client that went away) aborts the request."""
        p = self._enqueue(prompt, max_new, stream=True, stop_ids=stop_ids, sampling=sampling, stop_strs=stop_strs,
                          detok=detok)
        try:
            while True:
                try:
                    item = p.stream.get(timeout=timeout)
                except queue.Empty:
                    raise TimeoutError("request timed out") from None
                if item is None:
                    break
                yield item
        finally:
            if not p.event.is_set():
                self.abort(p)
        if p.error is not None:
            raise RuntimeError(p.error)
        if reason_out is not None:
            reason_out.append(p.reason)

    def overloaded(self) -> bool:
        with self._live_lock:
            return self.max_queued is not None and self._live >= self.max_queued

    def _release_live(self):
        with self._live_lock:
            self._live -= 1

    def flush_cache(self):
        """Drop the prefix cache's unreferenced pages on every rank (rank 0)."""
        self.q.put(self.FLUSH)

    def abort(self, p):
        """End a submitted request early (rank 0, any thread): every rank drops
        it at the same step; its waiter gets the tokens so far."""
        if not p.abort_sent and not p.event.is_set():
            p.abort_sent = True
            self.q.put((self.ABORT, p.sid))

    def _enqueue_check(self, prompt, max_new):
        if not prompt:
            raise ValueError("empty prompt")
        if max_new < 1:
            raise ValueError("max_tokens must be at least 1")
        vocab = getattr(getattr(self.engine, "cfg", None), "vocab", None)
        if isinstance(vocab, int) and (min(prompt) < 0 or max(prompt) >= vocab):
            raise ValueError(f"prompt token ids must lie in [0, {vocab})")
        limit = self.max_prompt
        cap = getattr(self.engine, "max_request_tokens", None)
        if isinstance(cap, int):
            limit = cap if limit is None else min(limit, cap)
        if limit is not None and len(prompt) + max_new > limit:
            raise ValueError(f"prompt + max_tokens = {len(prompt) + max_new} exceeds the engine's "
                             f"max sequence {limit}")

    def _enqueue(self, prompt, max_new, stream, stop_ids=None, sampling=None, stop_strs=(), detok=None, logprobs=None,
                 prompt_logprobs=False):
        if self._stopped.is_set():
            raise RuntimeError("server stopped")
        self._enqueue_check(prompt, max_new)
        with self._live_lock:
            if self.max_queued is not None and self._live >= self.max_queued:
                raise Overloaded(f"{self._live} requests in flight (limit {self.max_queued})")
            self._live += 1
        stop_strs = tuple(x for x in stop_strs if x)
        if stop_strs and detok is None:
            raise ValueError("stop strings need a detokenizer")
        p = _Pending(list(prompt), int(max_new), stream=stream,
                     stop_ids=self.stop_ids if stop_ids is None else stop_ids, sampling=sampling,
                     sid=next(self._sids), stop_strs=stop_strs, detok=detok, logprobs=logprobs,
                     prompt_logprobs=prompt_logprobs)
        p.on_finish = self._release_live
        self.q.put(p)
        return p

    def stop(self):
        """Ask every rank's loop to exit after the current step (rank 0)."""
        self.q.put(self.SHUTDOWN)

    # ------------------------------------------------------------ every rank
    def _next_commands(self, idle: bool):
        """Rank 0: the requests that arrived since the last step (blocking
        while the engine is idle); every rank: the same list."""
        cmds = []
        if self.rank == 0:
            if idle:
                cmds.append(self.q.get())  # nothing to run: wait for work
            while True:
                try:
                    cmds.append(self.q.get_nowait())
                except queue.Empty:
                    break
        if self.world > 1:
            import torch.distributed as dist

            if not idle and self._fast is not None:
                # every rank is here within one engine step: share the count
                ar, cnt = self._fast
                cnt.zero_()
                if self.rank == 0:
                    cnt[0] = float(len(cmds))
                self.stats["control_shm"] += 1
                if int(ar.all_reduce(cnt)[0].item()) == 0:
                    return cmds  # nothing new (rank 0's list is empty too)
            self.stats["control_gloo"] += 1
            payload = [[c if not isinstance(c, _Pending) else
                        (c.sid, c.prompt, c.max_new, c.stop_ids, c.sampling, c.logprobs, c.prompt_logprobs)
                        for c in cmds]]
            dist.broadcast_object_list(payload, src=0, group=self.group)
            if self.rank != 0:
                cmds = [c if isinstance(c, str) or c[0] == self.ABORT else
                        _Pending(c[1], c[2], stop_ids=c[3], sampling=c[4], sid=c[0], logprobs=c[5],
                                 prompt_logprobs=c[6]) for c in payload[0]]
        return cmds

    def serve_forever(self):
        eng = self.engine
        try:
            while True:
                idle = not eng.sched.has_work()
                cmds = self._next_commands(idle)
                stop = False
                for c in cmds:
                    if c == self.SHUTDOWN:
                        stop = True
                        continue
                    if c == self.FLUSH:  # every rank, same step
                        pc = getattr(eng, "prefix_cache", None)
                        if pc is not None:
                            pc.flush()
                        continue
                    if isinstance(c, tuple):  # (ABORT, sid): the same request on every rank
                        rid = self._rid_of_sid.get(c[1])
                        if rid is not None:
                            eng.abort(rid)
                        continue
                    try:
                        extra = {} if c.logprobs is None else {"logprobs": c.logprobs}
                        if c.prompt_logprobs:
                            extra["prompt_logprobs"] = True
                        if c.sampling is None:
                            req = eng.add_request(c.prompt, c.max_new, c.stop_ids, **extra)
                        else:
                            from .engine.sampling import SamplingParams

                            req = eng.add_request(c.prompt, c.max_new, c.stop_ids, SamplingParams(*c.sampling),
                                                  **extra)
                    except ValueError as e:
                        # rejected on every rank alike (same command, same engine
                        # state): fail this request only
                        c.finish(error=e)
                        continue
                    c.req = req
                    self._by_rid[req.rid] = c
                    self._rid_of_sid[c.sid] = req.rid
                    self.stats["requests"] += 1
                    self.stats["prompt_tokens"] += len(c.prompt)
                if stop:
                    break
                if eng.sched.has_work():
                    eng.step()
                    self.stats["steps"] += 1
                if self.rank == 0:
                    for p in self._by_rid.values():  # stream tokens as they appear
                        if p.stream is not None and p.req is not None and len(p.req.output) > p.sent:
                            p.stream.put(list(p.req.output[p.sent:]))
                            p.sent = len(p.req.output)
                        if p.stop_strs and p.req is not None and len(p.req.output) > p.checked:
                            p.checked = len(p.req.output)
                            # a new match ends in the newest tokens: decode a tail
                            # window, not the whole output, every step
                            win = max(16, 4 * max(len(x) for x in p.stop_strs))
                            if _find_stop(p.detok(p.req.output[-win:]), p.stop_strs) >= 0:
                                p.stop_hit = True
                                self.abort(p)  # every rank drops it next step
                done, eng.sched.finished = eng.sched.finished, []
                for r in done:
                    p = self._by_rid.pop(r.rid, None)
                    if p is not None:
                        self._rid_of_sid.pop(p.sid, None)
                        self.stats["completion_tokens"] += len(r.output)
                        times = getattr(r, "token_times", None) or []
                        if times and getattr(r, "t_arrive", 0):
                            self.ttft.append(times[0] - r.t_arrive)
                            self.itl.extend(b - a for a, b in zip(times, times[1:]))
                        if self.log_requests and self.rank == 0:
                            t0 = getattr(r, "t_arrive", 0) or 0
                            logger.info("request %s", json.dumps({
                                "id": p.sid, "prompt_tokens": len(p.prompt), "output_tokens": len(r.output),
                                "finish_reason": getattr(r, "finish_reason", None),
                                "ttft_ms": round((times[0] - t0) * 1e3, 3) if times and t0 else None,
                                "e2e_ms": round((time.perf_counter() - t0) * 1e3, 3) if t0 else None}))
                        out = list(r.output)
                        p.reason = getattr(r, "finish_reason", None) or "length"
                        if p.stop_strs and p.detok is not None:
                            k = _stop_prefix(out, p.stop_strs, p.detok)
                            if k is not None:
                                out, p.reason = out[:k], "stop"
                        p.token_logprobs = list(getattr(r, "token_logprobs", None) or [])[:len(out)]
                        p.prompt_token_logprobs = list(getattr(r, "prompt_token_logprobs", None) or [])
                        p.finish(output=out)
        except BaseException as e:  # noqa: BLE001 - fail every waiter, then re-raise
            for p in self._by_rid.values():
                p.finish(error=repr(e))
            raise
        finally:
            self._stopped.set()
            if self._fast is not None:
                self._fast[0].close()
                self._fast = None
            for p in self._by_rid.values():
                if not p.event.is_set():
                    p.finish(error="server stopped")
            while True:
                try:
                    c = self.q.get_nowait()
                except queue.Empty:
                    break
                if isinstance(c, _Pending):
                    c.finish(error="server stopped")


def _find_stop(text: str, stops) -> int:
    """Index of the earliest stop string in ``text``, or -1."""
    hits = [i for i in (text.find(x) for x in stops) if i >= 0]
    return min(hits) if hits else -1


def _held_back(text: str, stops) -> int:
    """Characters at the end of ``text`` that could begin a stop string (a
    stream holds them until the next tokens decide)."""
    hold = 0
    for x in stops:
        for k in range(min(len(x) - 1, len(text)), hold, -1):
            if text.endswith(x[:k]):
                hold = k
                break
    return hold


def _stop_prefix(tokens, stops, detok):
    """Length of the shortest token prefix whose text contains a stop string
    (None if the whole output holds none)."""
    if _find_stop(detok(tokens), stops) < 0:
        return None
    k = len(tokens)
    while k > 1 and _find_stop(detok(tokens[:k - 1]), stops) >= 0:
        k -= 1
    return k


def build_app(server: EngineServer, model_name: str, tokenizer=None, api_key: str = None):
    """FastAPI app with /health, /metrics, /v1/models, /v1/completions,
    /v1/chat/completions and /generate (plain or streamed; greedy or
    sampled; stop token ids and stop strings). ``api_key``: requests to the
    model endpoints need ``Authorization: Bearer <api_key>`` (/health and
    /metrics stay open for probes)."""
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
            if request.url.path not in ("/health", "/metrics"):
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
        ids_ = body.get("stop_token_ids")
        return None if ids_ is None else [int(t) for t in ids_]

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

    def _run(prompt, max_tokens, stop=None, sampling=None, stops=(), logprobs=None, prompt_logprobs=False):
        """(output ids, finish reason, per-token logprobs, prompt logprobs)."""
        try:
            p = server._submit_pending(prompt, max_tokens, stop_ids=stop, sampling=sampling, stop_strs=stops,
                                       detok=tok.decode, logprobs=logprobs, prompt_logprobs=prompt_logprobs)
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

    def _sse(prompt, max_tokens, chunk_of, stop=None, sampling=None, stops=()):
        """Server-sent events: one chunk per engine step's new tokens (the text
        delta of the decoded output, cut before a stop string), a last chunk
        with finish_reason and usage, then [DONE]. A client that disconnects
        closes the generator, which aborts the request."""
        def gen():
            out, reason, sent = [], [], ""
            fin = None
            try:
                stream = server.submit_stream(prompt, max_tokens, stop_ids=stop, reason_out=reason,
                                              sampling=sampling, stop_strs=stops, detok=tok.decode)
                try:
                    for toks in stream:
                        out += toks
                        hit = bool(stops) and _find_stop(tok.decode(out), stops) >= 0
                        text = _text(out, stops)
                        if stops and not hit:
                            text = text[:len(text) - _held_back(text, stops)]
                        delta, sent = text[len(sent):], text
                        yield "data: " + json.dumps(chunk_of(toks, delta, None, None)) + "\n\n"
                        if hit:
                            fin = "stop"  # the server loop drops the request on every rank
                            break
                finally:
                    stream.close()
                fin = fin or (reason[0] if reason else "length")
                if fin == "stop" and stops:
                    out = out[:_stop_prefix(out, stops, tok.decode) or len(out)]
                rest = _text(out, stops)[len(sent):]  # text held back for a stop string that never came
                yield "data: " + json.dumps(chunk_of([], rest, fin, _usage(prompt, out))) + "\n\n"
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
        if body.get("stream"):
            _n(body)
            if len(prompts) > 1:
                raise HTTPException(400, "several prompts are not supported with stream")
            _check(prompt, max_tokens)
            cid, created = f"cmpl-{next(ids)}", int(time.time())
            return _sse(prompt, max_tokens, lambda toks, text, fin, usage: {
                "id": cid, "object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "text": text, "token_ids": toks, "finish_reason": fin}],
                **({"usage": usage} if usage else {})}, stop, _sampling(body), stops)
        lp = body.get("logprobs")
        lp = None if lp is None or lp is False else int(lp)
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
        if body.get("stream"):
            _n(body)
            _check(prompt, max_tokens)
            cid, created = f"chatcmpl-{next(ids)}", int(time.time())
            return _sse(prompt, max_tokens, lambda toks, text, fin, usage: {
                "id": cid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                "choices": [{"index": 0, "delta": {"content": text} if (toks or text) else {},
                             "token_ids": toks, "finish_reason": fin}],
                **({"usage": usage} if usage else {})}, stop, _sampling(body), stops)
        lp = int(body.get("top_logprobs") or 0) if body.get("logprobs") else None
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
        ``stream`` the same objects, cumulative, as server-sent events."""
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
            return {"text": _text(out, stops), "output_ids": out, "meta_info": meta}

        if body.get("stream"):
            _check(prompt, max_new)

            def gen():
                out, reason = [], []
                try:
                    stream = server.submit_stream(prompt, max_new, stop_ids=stop, reason_out=reason,
                                                  sampling=sampling, stop_strs=stops, detok=tok.decode)
                    fin = None
                    try:
                        for toks in stream:
                            out += toks
                            if stops and _find_stop(tok.decode(out), stops) >= 0:
                                fin = "stop"
                                break
                            yield "data: " + json.dumps(result(out, None)) + "\n\n"
                    finally:
                        stream.close()
                    fin = fin or (reason[0] if reason else "length")
                    if fin == "stop" and stops:
                        out = out[:_stop_prefix(out, stops, tok.decode) or len(out)]
                    yield "data: " + json.dumps(result(out, fin)) + "\n\n"
                except (RuntimeError, TimeoutError) as e:
                    yield "data: " + json.dumps({"error": {"message": str(e)}}) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(iterate_in_threadpool(gen()), media_type="text/event-stream")
        out, fin, lps, plps = await run_in_threadpool(_run, prompt, max_new, stop, sampling, stops,
                                                      top_n if want_lp else None, score_prompt)
        return result(out, fin, lps, plps)

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


RANDOM_MODELS = ("8b", "70b", "tiny")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
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
    return __package__ or __name__.rsplit(".", 1)[0]


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
    from .router import Router, build_router_app

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
    tp = par.TPGroup(None, dev, use_mailbox=False if args.impl == "oracle" else None) if world > 1 else None
    ctrl = dist.new_group(backend="gloo", timeout=datetime.timedelta(days=7)) if world > 1 else None
    opts = dict(max_batch=args.max_batch, chunk=args.chunk, use_graphs=not args.no_graphs,
                impl=args.impl, prefill_graph=(args.impl == "native" and not args.no_graphs),
                prefix_cache=args.prefix_cache, mem_fraction=args.mem_fraction, mixed_chunk=args.mixed_chunk,
                schedule_policy=args.schedule_policy or ("lpm" if args.prefix_cache else "fcfs"))
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
                                                **opts)
        cfg = eng.cfg
        tokenizer = eng.tokenizer
        if tokenizer is None:  # token-id prompts still work
            logger.warning("no tokenizer in %s; using the byte tokenizer", model_path)
        elif args.chat_template:
            tokenizer.tok.chat_template = load_chat_template(args.chat_template)
    else:
        cfg = models.LlamaConfig.by_name(name)
        opts.setdefault("max_seq", min(16384, cfg.max_pos))
        eng = eng_mod.LLMEngine(cfg, tp=tp, device=dev, **opts)
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


if __name__ == "__main__":
    main()
