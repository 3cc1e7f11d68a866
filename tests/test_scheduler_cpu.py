"""Chunked-prefill scheduler, block allocator and KV slot mapping on CPU.

The policy under test is sglang's default, which the reference relies on
for its chunk-1024/2048 prefill measurements (docs/performance.md:29-49):
prefill chunks first, in arrival order, a chunk may span the tail of one
prompt and the head of the next; otherwise every running request decodes.
"""
import importlib

import pytest

sched_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine.scheduler")
kv_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine.kv_cache")
PAGE = kv_mod.PAGE


def _req(rid, n, max_new):
    return sched_mod.Request(rid=rid, prompt=list(range(n)), max_new=max_new)


def _drive(s, tok=7):
    """Run the scheduler to completion with a constant next token; returns
    the batch sequence as (kind, [(rid, start, n)] or [rids])."""
    trace = []
    while s.has_work():
        b = s.next_batch()
        if b.kind == "prefill":
            trace.append(("prefill", [(p.req.rid, p.start, p.n) for p in b.pieces]))
            s.after_prefill(b, [tok] * len(b.pieces))
        else:
            trace.append(("decode", [r.rid for r in b.reqs]))
            s.after_decode(b, [tok] * len(b.reqs))
    return trace


def test_chunks_span_prompts_in_arrival_order():
    s = sched_mod.Scheduler(chunk=100, max_batch=8)
    for rid, n in enumerate((150, 30, 70)):
        s.add(_req(rid, n, 2))
    trace = _drive(s)
    assert trace[0] == ("prefill", [(0, 0, 100)])
    assert trace[1] == ("prefill", [(0, 100, 50), (1, 0, 30), (2, 0, 20)])
    assert trace[2] == ("prefill", [(2, 20, 50)])
    # every prompt done: one decode step for all three (max_new=2: 1 token from prefill + 1 decode)
    assert trace[3] == ("decode", [0, 1, 2])
    assert len(trace) == 4
    assert [len(r.output) for r in sorted(s.finished, key=lambda r: r.rid)] == [2, 2, 2]


def test_prefill_has_priority_over_decode():
    s = sched_mod.Scheduler(chunk=64, max_batch=8)
    s.add(_req(0, 10, 5))
    b = s.next_batch()
    s.after_prefill(b, [1])
    assert s.next_batch().kind == "decode"
    s.add(_req(1, 100, 2))  # arrives while request 0 decodes
    b = s.next_batch()
    assert b.kind == "prefill" and b.pieces[0].req.rid == 1 and b.pieces[0].n == 64


def test_admission_limited_by_batch_slots_and_kv_blocks():
    alloc = kv_mod.BlockAllocator(num_blocks=1 + 10)  # block 0 reserved
    s = sched_mod.Scheduler(chunk=1000, max_batch=2, allocator=alloc)
    for rid in range(3):
        s.add(_req(rid, 40, 8))  # 48 tokens -> 3 blocks each
    b = s.next_batch()
    assert [p.req.rid for p in b.pieces] == [0, 1]  # only 2 batch slots
    assert alloc.free == 10 - 6
    s.after_prefill(b, [1, 1])
    trace = _drive(s)
    assert any(k == "prefill" and pieces[0][0] == 2 for k, pieces in trace)  # admitted once a slot freed
    assert alloc.free == 10 and len(s.finished) == 3
    # blocks never overlap between requests alive at the same time, and block 0 is never handed out
    alloc2 = kv_mod.BlockAllocator(num_blocks=9)
    got = [alloc2.alloc(4), alloc2.alloc(4)]
    assert 0 not in got[0] + got[1] and len(set(got[0] + got[1])) == 8
    with pytest.raises(MemoryError):
        alloc2.alloc(1)


def test_kv_memory_admission_waits_instead_of_failing():
    alloc = kv_mod.BlockAllocator(num_blocks=1 + 4)
    s = sched_mod.Scheduler(chunk=1000, max_batch=8, allocator=alloc)
    s.add(_req(0, 50, 14))  # 64 tokens = 4 blocks: the whole cache
    s.add(_req(1, 10, 2))
    b = s.next_batch()
    assert [p.req.rid for p in b.pieces] == [0]
    s.after_prefill(b, [1])
    assert s.next_batch().kind == "decode"  # request 1 waits for blocks
    _drive(s)
    assert sorted(r.rid for r in s.finished) == [0, 1] and alloc.free == 4


def test_request_longer_than_max_seq_is_rejected():
    s = sched_mod.Scheduler(chunk=64, max_batch=2, max_seq=100)
    with pytest.raises(ValueError):
        s.add(_req(0, 90, 20))


def test_slots_map_positions_to_pages():
    blocks = [5, 9, 2]
    slots = kv_mod.PagedKVCache.slots(None, blocks, 14, 5)
    assert slots == [5 * PAGE + 14, 5 * PAGE + 15, 9 * PAGE + 0, 9 * PAGE + 1, 9 * PAGE + 2]
    assert kv_mod.PagedKVCache.blocks_for(33) == 3
    assert kv_mod.PagedKVCache.bytes_per_token(32, 8, 128) == 32 * 2 * 8 * 128 * 2


def test_stop_token_ends_generation():
    s = sched_mod.Scheduler(chunk=64, max_batch=4)
    a = sched_mod.Request(rid=0, prompt=[1, 2, 3], max_new=10, stop_ids=(99,))
    b = sched_mod.Request(rid=1, prompt=[4, 5], max_new=3)
    s.add(a)
    s.add(b)
    batch = s.next_batch()
    s.after_prefill(batch, [7, 7])
    toks = iter([[8, 8], [99, 9]])
    while s.has_work():
        batch = s.next_batch()
        s.after_decode(batch, next(toks)[:len(batch.reqs)])
    assert a.output == [7, 8, 99] and a.finish_reason == "stop"     # stops on (and keeps) the stop id
    assert b.output == [7, 8, 9] and b.finish_reason == "length"
    # a stop id produced by the prefill itself ends the request at once
    s2 = sched_mod.Scheduler(chunk=64, max_batch=4)
    c = sched_mod.Request(rid=2, prompt=[1], max_new=5, stop_ids=(7,))
    s2.add(c)
    s2.after_prefill(s2.next_batch(), [7])
    assert not s2.has_work() and c.output == [7] and c.finish_reason == "stop"


def _pc_sched(num_blocks=64, chunk=1000, max_batch=8):
    alloc = kv_mod.BlockAllocator(num_blocks=num_blocks)
    pc = kv_mod.PrefixCache(alloc)
    return sched_mod.Scheduler(chunk=chunk, max_batch=max_batch, allocator=alloc, prefix_cache=pc), pc, alloc


def _run_one(s, req, tok=7):
    s.add(req)
    while s.has_work():
        b = s.next_batch()
        if b.kind == "prefill":
            s.after_prefill(b, [tok] * len(b.pieces))
        else:
            s.after_decode(b, [tok] * len(b.reqs))


def test_prefix_cache_shares_full_pages_of_a_common_prefix():
    s, pc, alloc = _pc_sched()
    common = list(range(100, 140))                      # 40 tokens: 2 full pages + 8
    a = sched_mod.Request(rid=0, prompt=common + [1, 2, 3], max_new=2)
    s.add(a)
    first = s.next_batch()
    a_blocks = list(a.blocks)
    s.after_prefill(first, [7])
    while s.has_work():
        s.after_decode(s.next_batch(), [7])
    free_after_a = alloc.free
    assert pc.evictable == 2                            # a's 2 full prompt pages stay cached
    b = sched_mod.Request(rid=1, prompt=common + [9] * 30, max_new=2)
    s.add(b)
    batch = s.next_batch()
    assert b.cached_pages == 2 and b.computed == 32     # prefill starts after the shared pages
    assert batch.pieces[0].start == 32 and batch.pieces[0].n == len(b.prompt) - 32
    assert b.blocks[:2] == a_blocks[:2]                 # the same physical pages
    assert pc.evictable == 0 and pc.hits == 2           # referenced again
    s.after_prefill(batch, [5])
    while s.has_work():
        s.after_decode(s.next_batch(), [5])
    # b registered its own 2 further full pages (common + 30 = 70 tokens -> 4 full pages)
    assert pc.evictable == 4 and alloc.free == free_after_a - 2


def test_prefix_cache_never_shares_the_page_of_the_last_token():
    s, pc, _ = _pc_sched()
    p = list(range(32))                                 # exactly 2 full pages
    _run_one(s, sched_mod.Request(rid=0, prompt=p, max_new=1))
    again = sched_mod.Request(rid=1, prompt=p, max_new=1)
    s.add(again)
    b = s.next_batch()
    assert again.cached_pages == 1 and b.pieces[0].start == 16 and b.pieces[0].n == 16


def test_prefix_cache_evicts_lru_pages_when_memory_is_short():
    s, pc, alloc = _pc_sched(num_blocks=1 + 6)
    _run_one(s, sched_mod.Request(rid=0, prompt=list(range(48)), max_new=1))   # 3 full pages cached
    assert pc.evictable == 3 and alloc.free == 3
    big = sched_mod.Request(rid=1, prompt=list(range(1000, 1080)), max_new=1)  # needs 6 blocks
    _run_one(s, big)
    assert big.done and big.cached_pages == 0
    assert sorted(pc.ref.values()) == [0] * len(pc.ref)  # nothing referenced after both finished


def test_prefix_cache_checks_tokens_not_just_hashes():
    s, pc, _ = _pc_sched()
    p = list(range(40))
    _run_one(s, sched_mod.Request(rid=0, prompt=p, max_new=1))
    # poison the table entry's stored tokens: a hash hit with different tokens must miss
    key = next(iter(pc.table))
    blk, page = pc.table[key]
    pc.table[key] = (blk, tuple(t + 1 for t in page))
    r = sched_mod.Request(rid=1, prompt=p, max_new=1)
    s.add(r)
    s.next_batch()
    assert r.cached_pages == 0


def test_request_larger_than_the_whole_kv_cache_is_rejected_not_queued():
    alloc = kv_mod.BlockAllocator(num_blocks=1 + 4)          # 64 tokens of cache
    s = sched_mod.Scheduler(chunk=64, max_batch=2, allocator=alloc, max_seq=1000)
    assert alloc.capacity == 4
    with pytest.raises(ValueError, match="KV cache"):
        s.add(_req(0, 60, 20))                               # 80 tokens: it would wait forever
    s.add(_req(1, 50, 14))                                   # exactly 64 tokens fits
    assert len(s.waiting) == 1


def test_kv_blocks_for_a_memory_fraction():
    GB = 1 << 30
    block = kv_mod.PagedKVCache.bytes_per_token(32, 8, 128) * PAGE       # 8B at TP=1: 2 MiB per page
    assert block == 2 << 20
    # 180 GB device, 16 GB already used by weights, weights + cache within 90 %
    n = kv_mod.PagedKVCache.blocks_for_memory(180 * GB, 164 * GB, 0.9, block)
    assert n == int((0.9 * 180 * GB - 16 * GB) // block)
    assert kv_mod.PagedKVCache.blocks_for_memory(180 * GB, 10 * GB, 0.9, block) == 0   # nothing left


def test_request_needs_a_prompt_and_a_positive_budget():
    s = sched_mod.Scheduler(chunk=64, max_batch=2)
    for prompt, max_new in (([], 4), ([1, 2], 0), ([1, 2], -3)):
        with pytest.raises(ValueError):
            s.add(sched_mod.Request(rid=0, prompt=prompt, max_new=max_new))


def test_abort_frees_pages_and_slots_wherever_the_request_is():
    alloc = kv_mod.BlockAllocator(num_blocks=1 + 40)
    pc = kv_mod.PrefixCache(alloc)
    s = sched_mod.Scheduler(chunk=32, max_batch=2, allocator=alloc, prefix_cache=pc)
    reqs = [_req(i, 40, 8) for i in range(3)]
    for r in reqs:
        s.add(r)
    b = s.next_batch()                               # 0 and 1 admitted (2 slots), 2 waits
    assert [p.req.rid for p in b.pieces] == [0] and len(s.waiting) == 1
    s.after_prefill(b, [7])
    assert s.abort(2) and reqs[2].finish_reason == "abort" and reqs[2].output == []   # from the queue
    assert s.abort(1) and reqs[1].blocks == [] and reqs[1].slot == -1                 # mid-prefill
    while reqs[0].computed < 40:
        s.after_prefill(s.next_batch(), [7])
    s.after_decode(s.next_batch(), [5])
    assert s.abort(0) and reqs[0].output == [7, 5] and reqs[0].finish_reason == "abort"  # decoding
    assert not s.has_work() and not s.abort(0)
    assert sorted(r.rid for r in s.finished) == [0, 1, 2]
    assert alloc.free + pc.evictable == 40                                           # every page back
    assert sorted(s._free_slots) == [0, 1]


def test_mixed_chunks_carry_decode_tokens_while_prompts_prefill():
    s = sched_mod.Scheduler(chunk=16, max_batch=4, mixed=True)
    a = sched_mod.Request(rid=0, prompt=[1] * 5, max_new=6)
    s.add(a)
    s.after_prefill(s.next_batch(), [7])                     # a is decoding now
    b = sched_mod.Request(rid=1, prompt=[2] * 40, max_new=2)
    s.add(b)
    kinds = []
    while b.computed < 40:
        batch = s.next_batch()
        assert batch.kind == "prefill"
        dec = [p for p in batch.pieces if p.decode]
        kinds.append(len(dec))
        assert all(p.req is a and p.n == 1 and p.start == a.total_len - 1 and p.tokens() == [a.output[-1]]
                   for p in dec)
        s.after_prefill(batch, [8] * len(batch.pieces))
    assert kinds == [1, 1, 1]                                # a decoded in each of b's three chunks
    assert a.output == [7, 8, 8, 8] and a.computed == 5 + 3
    while s.has_work():
        batch = s.next_batch()
        s.after_decode(batch, [9] * len(batch.reqs))
    assert a.output == [7, 8, 8, 8, 9, 9] and b.output == [8, 9]


def test_lpm_admits_the_longest_cached_prefix_first():
    s, pc, alloc = _pc_sched(num_blocks=64, chunk=1000, max_batch=1)
    s.policy = "lpm"
    shared = list(range(500, 548))                                   # 3 full pages
    _run_one(s, sched_mod.Request(rid=0, prompt=shared + [1], max_new=1))
    cold = sched_mod.Request(rid=1, prompt=list(range(2000, 2040)), max_new=1)
    warm = sched_mod.Request(rid=2, prompt=shared + [7, 8], max_new=1)
    s.add(cold)
    s.add(warm)
    b = s.next_batch()                                               # one slot: lpm picks the cache hit
    assert b.pieces[0].req is warm and warm.cached_pages == 3
    fcfs, _, _ = _pc_sched(num_blocks=64, chunk=1000, max_batch=1)
    fcfs.add(sched_mod.Request(rid=3, prompt=[1] * 20, max_new=1))
    fcfs.add(sched_mod.Request(rid=4, prompt=[2] * 20, max_new=1))
    assert fcfs.next_batch().pieces[0].req.rid == 3                  # arrival order by default
    with pytest.raises(ValueError):
        sched_mod.Scheduler(policy="random")


def test_prefix_cache_flush_keeps_pages_in_use():
    s, pc, alloc = _pc_sched(num_blocks=64)
    _run_one(s, sched_mod.Request(rid=0, prompt=list(range(48)), max_new=1))     # 3 cached, unreferenced
    held = sched_mod.Request(rid=1, prompt=list(range(1000, 1040)), max_new=4)
    s.add(held)
    s.after_prefill(s.next_batch(), [1])                                       # 2 more cached, referenced
    assert pc.evictable == 3
    assert pc.flush() == 3 and pc.evictable == 0
    assert len(pc.table) == 2 and all(v == 1 for v in pc.ref.values())         # the live request's pages stay
    while s.has_work():
        s.after_decode(s.next_batch(), [1])
    assert alloc.free + pc.evictable == alloc.capacity
