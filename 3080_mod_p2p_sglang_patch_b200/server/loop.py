"""The lockstep request loop of the TP ranks (rank 0 owns the queue and
broadcasts each step's commands; every rank steps the same engine), with
stop-string, abort and overload handling."""
import collections
import itertools
import json
import logging
import queue
import threading
import time

from ..engine.stops import find_stop as _find_stop  # noqa: F401 - also used by http.py
from ..engine.stops import held_back as _held_back  # noqa: F401
from ..engine.stops import stop_prefix as _stop_prefix
from ..engine.stops import tail_hit

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
        self._named = {}                 # rank 0: client request id (sglang's ``rid``) -> live request
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

            from ..config import CommConfig
            from ..parallel.communicator import MailboxAR

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
                        logprobs=None, prompt_logprobs=False, name=None):
        """``submit`` returning the finished request record (output, reason,
        token_logprobs, prompt_token_logprobs). ``name``: a client request id
        that ``abort_request`` can end the request by."""
        p = self._enqueue(prompt, max_new, stream=False, stop_ids=stop_ids, sampling=sampling, stop_strs=stop_strs,
                          detok=detok, logprobs=logprobs, prompt_logprobs=prompt_logprobs, name=name)
        if not p.event.wait(timeout):
            raise TimeoutError("request timed out")
        if isinstance(p.error, ValueError):  # the engine rejected the request itself
            raise p.error
        if p.error is not None:
            raise RuntimeError(p.error)
        return p

    def submit_stream(self, prompt: list, max_new: int, timeout: float = None, stop_ids=None, reason_out=None,
                      sampling=None, stop_strs=(), detok=None, name=None, logprobs=None):
        """Like ``submit`` but yields lists of new token ids as the engine
        produces them (rank 0, from an HTTP thread); the finish reason is
        appended to ``reason_out`` (a list) at the end. Closing the generator
        early (a client that went away) aborts the request. With ``logprobs``
        (k alternatives) it yields ``(token ids, logprobs)`` pairs instead, one
        ``(logprob, [(id, logprob)] * k)`` per token."""
        p = self._enqueue(prompt, max_new, stream=True, stop_ids=stop_ids, sampling=sampling, stop_strs=stop_strs,
                          detok=detok, name=name, logprobs=logprobs)
        try:
            while True:
                try:
                    item = p.stream.get(timeout=timeout)
                except queue.Empty:
                    raise TimeoutError("request timed out") from None
                if item is None:
                    break
                yield item if logprobs is not None else item[0]
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

    def abort_request(self, name) -> bool:
        """End the live request submitted with client id ``name`` (rank 0, any
        thread); False when no such request is in flight."""
        with self._live_lock:
            p = self._named.get(name)
        if p is None:
            return False
        self.abort(p)
        return True

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
                 prompt_logprobs=False, name=None):
        if self._stopped.is_set():
            raise RuntimeError("server stopped")
        self._enqueue_check(prompt, max_new)
        stop_strs = tuple(x for x in stop_strs if x)
        if stop_strs and detok is None:
            raise ValueError("stop strings need a detokenizer")
        p = _Pending(list(prompt), int(max_new), stream=stream,
                     stop_ids=self.stop_ids if stop_ids is None else stop_ids, sampling=sampling,
                     sid=next(self._sids), stop_strs=stop_strs, detok=detok, logprobs=logprobs,
                     prompt_logprobs=prompt_logprobs)
        with self._live_lock:
            if self.max_queued is not None and self._live >= self.max_queued:
                raise Overloaded(f"{self._live} requests in flight (limit {self.max_queued})")
            if name is not None and name in self._named:
                raise ValueError(f"request id {name!r} is already in flight")
            self._live += 1
            if name is not None:
                self._named[name] = p
        p.on_finish = self._release_live if name is None else (lambda: self._release_named(name))
        self.q.put(p)
        return p

    def _release_named(self, name):
        with self._live_lock:
            self._live -= 1
            self._named.pop(name, None)

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
                            from ..engine.sampling import SamplingParams

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
                            n = len(p.req.output)
                            lps = list(getattr(p.req, "token_logprobs", None) or [])[p.sent:n] \
                                if p.logprobs is not None else []
                            p.stream.put((list(p.req.output[p.sent:n]), lps))
                            p.sent = n
                        if p.stop_strs and p.req is not None and len(p.req.output) > p.checked:
                            p.checked = len(p.req.output)
                            # a new match ends in the newest tokens
                            if tail_hit(p.req.output, p.stop_strs, p.detok):
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
