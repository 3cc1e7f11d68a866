"""Request state and the chunked-prefill scheduler.

Policy (sglang's default): while any request still has prompt tokens to
prefill, the next batch is a prefill chunk of up to ``chunk`` tokens, taken
in admission order (a long prompt spans several chunks; a chunk may hold the
tail of one prompt and the head of the next). Otherwise all running requests
decode one token. With ``mixed`` a prefill batch also carries one decode
token of every running request. New requests are admitted while the running
set is below ``max_batch`` and the KV cache has room, in arrival order
("fcfs") or longest cached prefix first ("lpm"). ``abort`` ends a request
between steps.
"""
import collections
import dataclasses

from .kv_cache import PAGE


@dataclasses.dataclass
class Request:
    rid: int
    prompt: list
    max_new: int
    output: list = dataclasses.field(default_factory=list)
    blocks: list = dataclasses.field(default_factory=list)
    computed: int = 0          # tokens whose K/V are in the cache
    slot: int = -1             # row in the decode batch tables
    done: bool = False
    t_arrive: float = 0.0
    t_first: float = 0.0
    token_times: list = dataclasses.field(default_factory=list)
    # generation also ends after any of these token ids (e.g. the model's EOS);
    # the stop token is kept in the output
    stop_ids: tuple = ()
    finish_reason: str = None  # "length" or "stop" once done
    cached_pages: int = 0      # leading prompt pages served by the prefix cache
    sampling: object = None    # engine.sampling.SamplingParams (None = greedy)
    rng: object = None         # torch.Generator of a seeded sampled request
    # log-probabilities of the generated tokens: None = off, k >= 0 = each
    # token's logprob plus the k most likely alternatives
    logprobs: int = None
    # per generated token: (logprob, [(token id, logprob), ...] top-k)
    token_logprobs: list = dataclasses.field(default_factory=list)
    # logprobs of the prompt's own tokens (scoring; "echo"): one entry per
    # prompt token, None for the first (it has no context)
    prompt_logprobs: bool = False
    prompt_token_logprobs: list = dataclasses.field(default_factory=list)

    @property
    def sampled(self):
        return self.sampling is not None and not self.sampling.greedy

    @property
    def needs_logits(self):
        """Full logits are needed: a sampled request, or one that returns logprobs."""
        return (self.sampled or self.logprobs is not None or self.prompt_logprobs or
                (self.sampling is not None and self.sampling.adjusts))

    @property
    def total_len(self):
        return len(self.prompt) + len(self.output)

    @property
    def prefill_left(self):
        return len(self.prompt) - self.computed if self.computed < len(self.prompt) else 0


@dataclasses.dataclass
class PrefillPiece:
    req: Request
    start: int
    n: int
    # a running request's decode step carried by a prefill batch (mixed
    # chunks): one token, its last output, at position total_len - 1
    decode: bool = False

    @property
    def completes(self):
        """The piece's last row yields a token that is used."""
        return self.decode or self.start + self.n == len(self.req.prompt)

    def tokens(self):
        if self.decode:
            return [self.req.output[-1]]
        return self.req.prompt[self.start:self.start + self.n]


@dataclasses.dataclass
class Batch:
    kind: str  # "prefill" or "decode"
    pieces: list = None
    reqs: list = None

    @property
    def num_tokens(self):
        return sum(p.n for p in self.pieces) if self.kind == "prefill" else len(self.reqs)


class Scheduler:
    POLICIES = ("fcfs", "lpm")

    def __init__(self, chunk: int = 1024, max_batch: int = 64, allocator=None, max_seq: int = 16384,
                 prefix_cache=None, mixed: bool = False, policy: str = "fcfs"):
        if policy not in self.POLICIES:
            raise ValueError(f"schedule policy {policy!r}: {' | '.join(self.POLICIES)}")
        # admission order of waiting requests: "fcfs" (arrival) or "lpm" (the
        # longest cached prompt prefix first, ties by arrival; with a prefix
        # cache, as sglang's default)
        self.policy = policy
        self.chunk = chunk
        # mixed chunks (sglang's --enable-mixed-chunk): a prefill batch also
        # carries one decode token of every running request, so decoding does
        # not pause while long prompts prefill
        self.mixed = mixed
        self.max_batch = max_batch
        self.allocator = allocator
        self.max_seq = max_seq
        # kv_cache.PrefixCache (needs the allocator) or None
        self.prefix_cache = prefix_cache
        self.waiting = collections.deque()
        self.prefilling = []
        self.running = []
        self.finished = []
        self._free_slots = list(range(max_batch - 1, -1, -1))

    def add(self, req: Request):
        if not req.prompt or req.max_new < 1:
            raise ValueError(f"request {req.rid}: needs a prompt and max_new >= 1")
        n = len(req.prompt) + req.max_new
        if n > self.max_seq:
            raise ValueError(f"request {req.rid}: {len(req.prompt)}+{req.max_new} tokens exceed max_seq {self.max_seq}")
        if self.allocator is not None and (n + PAGE - 1) // PAGE > self.allocator.capacity:
            # it would wait for room forever
            raise ValueError(f"request {req.rid}: {n} tokens exceed the KV cache "
                             f"({self.allocator.capacity * PAGE} tokens)")
        self.waiting.append(req)

    def has_work(self):
        return bool(self.waiting or self.prefilling or self.running)

    def _admit(self):
        pc = self.prefix_cache
        if self.policy == "lpm" and pc is not None and len(self.waiting) > 1:
            # stable sort: equal matches keep their arrival order
            hits = {id(r): (0 if r.prompt_logprobs else len(pc.match(r.prompt, (len(r.prompt) - 1) // PAGE)))
                    for r in self.waiting}
            self.waiting = collections.deque(sorted(self.waiting, key=lambda r: -hits[id(r)]))
        while self.waiting and self._free_slots:
            req = self.waiting[0]
            need = (len(req.prompt) + req.max_new + PAGE - 1) // PAGE
            matched = []
            if pc is not None and not req.prompt_logprobs:  # scoring needs every position computed
                # full pages before the last prompt token (that one is always computed)
                matched = pc.match(req.prompt, (len(req.prompt) - 1) // PAGE)
            if self.allocator is not None:
                room = self.allocator.free + (pc.evictable if pc is not None else 0)
                if room < need - len(matched):
                    break
            self.waiting.popleft()
            if pc is not None:
                pc.acquire(matched)
                req.blocks = matched + pc.alloc_blocks(need - len(matched))
                req.computed = len(matched) * PAGE
                req.cached_pages = len(matched)
            elif self.allocator is not None:
                req.blocks = self.allocator.alloc(need)
            req.slot = self._free_slots.pop()
            self.prefilling.append(req)

    def next_batch(self):
        self._admit()
        if self.prefilling:
            budget = self.chunk
            pieces = []
            for req in self.prefilling:
                if budget <= 0:
                    break
                n = min(req.prefill_left, budget)
                if n <= 0:
                    continue
                pieces.append(PrefillPiece(req, req.computed, n))
                budget -= n
            if self.mixed:
                pieces.extend(PrefillPiece(r, r.total_len - 1, 1, decode=True) for r in self.running)
            return Batch("prefill", pieces=pieces)
        if self.running:
            return Batch("decode", reqs=list(self.running))
        return None

    def after_prefill(self, batch: Batch, next_tokens):
        """next_tokens: list aligned with batch.pieces (only completing pieces matter)."""
        for piece, tok in zip(batch.pieces, next_tokens):
            req = piece.req
            req.computed += piece.n
            if piece.decode:  # a running request's decode step
                req.output.append(int(tok))
                if self._done(req):
                    self.running.remove(req)
                    self._finish(req)
                continue
            if piece.completes:
                self.prefilling.remove(req)
                if self.prefix_cache is not None:
                    # the prompt's full pages now hold valid K/V: share them
                    self.prefix_cache.insert(req.prompt, req.blocks, req.cached_pages, len(req.prompt) // PAGE)
                req.output.append(int(tok))
                if self._done(req):
                    self._finish(req)
                else:
                    self.running.append(req)

    def after_decode(self, batch: Batch, next_tokens):
        for req, tok in zip(batch.reqs, next_tokens):
            req.computed += 1
            req.output.append(int(tok))
            if self._done(req):
                self.running.remove(req)
                self._finish(req)

    @staticmethod
    def _done(req):
        if req.stop_ids and req.output[-1] in req.stop_ids:
            req.finish_reason = "stop"
            return True
        if len(req.output) >= req.max_new:
            req.finish_reason = "length"
            return True
        return False

    def abort(self, rid: int) -> bool:
        """End request ``rid`` now, wherever it is (queued, prefilling or
        decoding): its pages and batch slot are released and it moves to
        ``finished`` with finish_reason "abort" and the tokens it has. Call
        between steps. False if no live request has that id."""
        for req in self.waiting:
            if req.rid == rid:
                self.waiting.remove(req)
                req.done, req.finish_reason = True, "abort"
                self.finished.append(req)
                return True
        for queue in (self.prefilling, self.running):
            for req in queue:
                if req.rid == rid:
                    queue.remove(req)
                    req.finish_reason = "abort"
                    self._finish(req)
                    return True
        return False

    def _finish(self, req):
        req.done = True
        if req.blocks:
            if self.prefix_cache is not None:
                self.prefix_cache.release(req.blocks)
            elif self.allocator is not None:
                self.allocator.release(req.blocks)
            req.blocks = []
        self._free_slots.append(req.slot)
        req.slot = -1
        self.finished.append(req)
