"""HTTP front end and the lockstep request loop, on CPU with a stand-in
engine (the real engine needs the GPU; tests/test_model_gpu.py covers it).

The reference's clients post OpenAI-style requests and read
``usage.prompt_tokens`` (tests/pp_bench.py:21-29); the same shapes are
checked here, plus that every TP rank runs the same requests in the same
order (two gloo ranks).
"""
import importlib
import os
import subprocess
import sys
import threading

import pytest

from _mp import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
srv_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.server")


class _Req:
    def __init__(self, rid, prompt, max_new):
        import time as _t

        self.rid, self.prompt, self.max_new, self.output = rid, list(prompt), max_new, []
        self.t_arrive, self.token_times = _t.perf_counter(), []


class _Sched:
    def __init__(self):
        self.running, self.finished = [], []

    def has_work(self):
        return bool(self.running)


class FakeEngine:
    """One token per running request per step: (sum(prompt) + len(output)) % 1000."""

    def __init__(self):
        self.sched = _Sched()
        self.n = 0
        self.log = []
        self.sampling_seen = []
        self.aborted = []   # (rid, steps taken when it was aborted)
        self.steps = 0

    def add_request(self, prompt, max_new, stop_ids=(), sampling=None, logprobs=None, prompt_logprobs=False):
        r = _Req(self.n, prompt, max_new)
        r.stop_ids = tuple(stop_ids)
        r.sampling = sampling
        r.logprobs, r.token_logprobs = logprobs, []
        # scoring: every prompt token after the first at -1.0
        r.prompt_token_logprobs = [None] + [(-1.0, [])] * (len(prompt) - 1) if prompt_logprobs else []
        self.sampling_seen.append(sampling)
        self.n += 1
        self.sched.running.append(r)
        self.log.append((r.rid, tuple(prompt), max_new))
        return r

    def abort(self, rid):
        for r in list(self.sched.running):
            if r.rid == rid:
                self.sched.running.remove(r)
                r.finish_reason = "abort"
                self.sched.finished.append(r)
                self.aborted.append((rid, self.steps))
                return True
        return False

    def step(self):
        import time as _t

        self.steps += 1
        for r in list(self.sched.running):
            r.output.append((sum(r.prompt) + len(r.output)) % 1000)
            if r.logprobs is not None:  # a fixed distribution: the token, then its successor
                t = r.output[-1]
                r.token_logprobs.append((-0.25, [(t, -0.25), (t + 1, -2.0)][:r.logprobs]))
            r.token_times.append(_t.perf_counter())
            r.finish_reason = "stop" if r.output[-1] in r.stop_ids else \
                ("length" if len(r.output) >= r.max_new else None)
            if r.finish_reason:
                self.sched.running.remove(r)
                self.sched.finished.append(r)


def expected(prompt, n):
    return [(sum(prompt) + i) % 1000 for i in range(n)]


def test_byte_tokenizer_roundtrip():
    tok = srv_mod.ByteTokenizer()
    text = "KV cache 页 16 ✓"
    ids = tok.encode(text)
    assert all(0 <= i < 256 for i in ids)
    assert tok.decode(ids) == text
    assert tok.decode(ids + [300, 4000]) == text  # ids >= 256 have no text


def test_http_completions_and_chat():
    requests = pytest.importorskip("requests")
    from conftest import free_port

    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    try:
        base = f"http://127.0.0.1:{port}"
        r = requests.post(base + "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4}, timeout=30)
        assert r.status_code == 200, r.text
        j = r.json()
        assert j["choices"][0]["token_ids"] == expected([5, 6, 7], 4)
        assert j["usage"] == {"prompt_tokens": 3, "completion_tokens": 4, "total_tokens": 7}
        # the reference's pp_bench request shape
        body = {"model": "fake", "messages": [{"role": "user", "content": "hello"}], "max_tokens": 1,
                "temperature": 0}
        r = requests.post(base + "/v1/chat/completions", json=body, timeout=30)
        assert r.status_code == 200, r.text
        j = r.json()
        prompt = srv_mod.ByteTokenizer().encode("<|user|>hello<|assistant|>")
        assert j["usage"]["prompt_tokens"] == len(prompt)
        assert j["choices"][0]["token_ids"] == expected(prompt, 1)
        # concurrent requests all complete
        outs = [None] * 8

        def client(i):
            outs[i] = requests.post(base + "/v1/completions", json={"prompt": [i + 1] * (i + 1), "max_tokens": i + 1},
                                    timeout=30).json()["choices"][0]["token_ids"]

        ths = [threading.Thread(target=client, args=(i,)) for i in range(8)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        for i in range(8):
            assert outs[i] == expected([i + 1] * (i + 1), i + 1)
        assert requests.post(base + "/v1/completions", json={"prompt": [], "max_tokens": 1}, timeout=30).status_code == 400
        assert requests.post(base + "/v1/completions", json={"prompt": [1] * 4096, "max_tokens": 8},
                             timeout=30).status_code == 400
        # stop_token_ids: prompt [10] generates 10, 11, 12, ...; stop at 12
        j = requests.post(base + "/v1/completions", json={"prompt": [10], "max_tokens": 8, "stop_token_ids": [12]},
                          timeout=30).json()
        assert j["choices"][0]["token_ids"] == [10, 11, 12] and j["choices"][0]["finish_reason"] == "stop"
        # sampling fields reach the engine as SamplingParams
        requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 1, "temperature": 0.7,
                                                      "top_p": 0.9, "top_k": 40, "seed": 5}, timeout=30)
        sp = eng.sampling_seen[-1]
        assert (sp.temperature, sp.top_k, sp.top_p, sp.seed) == (0.7, 40, 0.9, 5)
        assert eng.sampling_seen[0] is None  # greedy requests stay greedy
        h = requests.get(base + "/health", timeout=30).json()
        assert h["status"] == "ok" and h["requests"] == 12
        m = requests.get(base + "/metrics", timeout=30)
        assert m.status_code == 200 and m.headers["content-type"].startswith("text/plain")
        lines = m.text.splitlines()
        assert "mbx_requests_total 12" in lines
        assert any(ln.startswith('mbx_inter_token_latency_seconds{quantile="0.5"}') for ln in lines)
        assert any(ln.startswith("# TYPE mbx_generation_tokens_total counter") for ln in lines)
        assert "mbx_requests_in_flight 0" in lines and "mbx_num_running_reqs 0" in lines
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True
    assert not loop.is_alive()


def test_streaming_completions():
    """stream=true: server-sent events carry the tokens step by step, then
    a chunk with finish_reason and usage, then [DONE]."""
    requests = pytest.importorskip("requests")
    import json

    from conftest import free_port

    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    try:
        base = f"http://127.0.0.1:{port}"
        for path, body in (("/v1/completions", {"prompt": [3, 4], "max_tokens": 5, "stream": True}),
                           ("/v1/chat/completions", {"messages": [{"role": "user", "content": "x"}],
                                                     "max_tokens": 5, "stream": True})):
            r = requests.post(base + path, json=body, timeout=30, stream=True)
            assert r.status_code == 200 and r.headers["content-type"].startswith("text/event-stream")
            events = [ln[len("data: "):] for ln in r.iter_lines(decode_unicode=True) if ln.startswith("data: ")]
            assert events[-1] == "[DONE]"
            chunks = [json.loads(e) for e in events[:-1]]
            toks = [t for c in chunks for t in c["choices"][0]["token_ids"]]
            prompt = [3, 4] if path == "/v1/completions" else \
                srv_mod.ByteTokenizer().encode("<|user|>x<|assistant|>")
            assert toks == expected(prompt, 5)
            assert len(chunks) >= 3  # tokens arrive over several engine steps
            assert chunks[-1]["choices"][0]["finish_reason"] == "length"
            assert chunks[-1]["usage"]["completion_tokens"] == 5
        bad = requests.post(base + "/v1/completions", json={"prompt": [], "max_tokens": 1, "stream": True},
                            timeout=30)
        assert bad.status_code == 400
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def _lockstep(rank, world):
    import datetime

    import torch.distributed as dist

    ctrl = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, ctrl, rank, world)
    results = {}
    if rank == 0:
        def clients():
            ths = []
            for i in range(6):
                def one(i=i):
                    results[i] = server.submit([i, i + 1], 3 + i % 3, timeout=60)
                t = threading.Thread(target=one)
                t.start()
                ths.append(t)
            for t in ths:
                t.join()
            server.stop()

        threading.Thread(target=clients, daemon=True).start()
    server.serve_forever()
    return {"log": sorted(eng.log), "results": results, "stats": dict(server.stats)}


def test_lockstep_two_ranks():
    res = run_ranks(_lockstep, 2)
    assert res[0]["log"] == res[1]["log"] and len(res[0]["log"]) == 6
    # busy steps exchanged the command count over shared memory; gloo carried
    # only payloads and idle waits (same sequence on both ranks)
    st0, st1 = res[0]["stats"], res[1]["stats"]
    assert st0["control_shm"] > 0 and st0["control_shm"] == st1["control_shm"]
    assert st0["control_gloo"] == st1["control_gloo"] and st0["control_gloo"] <= 6 + 2
    for i, out in res[0]["results"].items():
        assert out == expected([i, i + 1], 3 + i % 3)


def test_cli_accepts_sglang_flag_spellings_and_model_dirs(tmp_path):
    p = srv_mod.build_parser()
    a = p.parse_args(["--model", str(tmp_path), "--tp-size", "2", "--chunked-prefill-size", "2048",
                      "--context-length", "8192", "--max-running-requests", "32", "--disable-cuda-graph"])
    assert (a.tp, a.chunk, a.max_seq, a.max_batch, a.no_graphs) == (2, 2048, 8192, 32, True)
    assert srv_mod.resolve_model(a) == (None, str(tmp_path))            # a directory is a checkpoint
    assert srv_mod.resolve_model(p.parse_args(["--model", "tiny"])) == ("tiny", None)
    assert srv_mod.resolve_model(p.parse_args(["--model-path", "/ck", "--model", "8b"])) == (None, "/ck")
    with pytest.raises(SystemExit):
        srv_mod.resolve_model(p.parse_args(["--model", str(tmp_path / "missing")]))


def test_tp_flag_relaunches_one_rank_per_gpu():
    for argv in (["--model", "tiny", "--tp", "4", "--port", "9"], ["--tp=4", "--model", "tiny", "--port", "9"],
                 ["--model", "tiny", "--tp-size", "4", "--port", "9"]):
        cmd = srv_mod.relaunch_command(argv, 4, 29555)
        assert cmd[1:3] == ["-m", "torch.distributed.run"]
        assert "--nproc-per-node=4" in cmd and "--master-addr=127.0.0.1" in cmd and "--master-port=29555" in cmd
        i = cmd.index("3080_mod_p2p_sglang_patch_b200.server")
        assert cmd[i - 1] == "-m" and sorted(cmd[i + 1:]) == sorted(["--model", "tiny", "--port", "9"])


def test_module_entry_point_runs_as_main():
    """``python -m <pkg>.server`` resolves the package's modules (``__name__``
    is ``__main__`` there); without a GPU it stops with a message, not a
    traceback."""
    env = dict(os.environ)
    env.pop("WORLD_SIZE", None)
    env["CUDA_VISIBLE_DEVICES"] = ""
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, "-m", "3080_mod_p2p_sglang_patch_b200.server", "--model", "tiny"],
                       capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert r.returncode == 1 and "needs a CUDA GPU" in r.stderr and "Traceback" not in r.stderr, r.stderr[-2000:]
    r = subprocess.run([sys.executable, "-m", "3080_mod_p2p_sglang_patch_b200.server", "--model", "nope"],
                       capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert r.returncode == 1 and "not a directory" in r.stderr


def test_pp_bench_against_the_server(capsys):
    """benchmarks/pp_bench.py (the reference's prefill benchmark method:
    max_tokens=1, usage.prompt_tokens / wall) against the HTTP front end."""
    import importlib.util

    from conftest import free_port

    spec = importlib.util.spec_from_file_location("pp_bench", os.path.join(ROOT, "benchmarks", "pp_bench.py"))
    pp = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(pp)
    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    try:
        res = pp.main(["--url", f"http://127.0.0.1:{port}", "--sizes", "300,120", "--warmup", "50"])
        assert [v["prompt_tokens"] for v in res.values()] == [300, 120]
        assert all(v["pp_tok_s"] > 0 for v in res.values())
        prompts = [p for _, p, _ in eng.log]
        assert len(prompts) == 3 and len({p[:4] for p in prompts}) == 3   # salted: no shared prefix
        assert all(m == 1 for _, _, m in eng.log)                          # max_tokens=1
        out = capsys.readouterr().out
        assert "SUMMARY " in out
        pp.main(["--url", f"http://127.0.0.1:{port}", "--sizes", "200", "--warmup", "20", "--text"])
        assert len(eng.log) == 5
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


class _PickyEngine(FakeEngine):
    """Rejects prompts that start with 999 the way the engine rejects a
    request its KV cache can never hold."""

    max_request_tokens = 64

    def add_request(self, prompt, max_new, stop_ids=(), sampling=None, **kw):
        if prompt and prompt[0] == 999:
            raise ValueError("too large for the KV cache")
        return super().add_request(prompt, max_new, stop_ids, sampling, **kw)


def test_engine_rejection_fails_one_request_and_the_server_keeps_serving():
    import requests

    from conftest import free_port

    eng = _PickyEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    url = f"http://127.0.0.1:{port}/v1/completions"
    try:
        r = requests.post(url, json={"prompt": [999, 1, 2], "max_tokens": 2}, timeout=60)
        assert r.status_code == 400 and "KV cache" in r.text
        r = requests.post(url, json={"prompt": list(range(1, 70)), "max_tokens": 2}, timeout=60)
        assert r.status_code == 400                       # beyond max_request_tokens: refused up front
        r = requests.post(url, json={"prompt": [5, 6], "max_tokens": 0}, timeout=60)
        assert r.status_code == 400                       # nothing to generate
        eng.cfg = type("Cfg", (), {"vocab": 100})()
        r = requests.post(url, json={"prompt": [5, 100], "max_tokens": 2}, timeout=60)
        assert r.status_code == 400 and "token ids" in r.text
        r = requests.post(url, json={"prompt": [5, 6], "max_tokens": 3}, timeout=60)
        assert r.status_code == 200 and r.json()["choices"][0]["token_ids"] == expected([5, 6], 3)
        assert loop.is_alive()
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def _serve(eng):
    from conftest import free_port

    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    return server, loop, http, f"http://127.0.0.1:{port}"


def test_stop_strings_end_generation_and_cut_the_text():
    """OpenAI ``stop``: the fake engine emits ids 100, 101, ... = bytes
    'd', 'e', 'f', 'g', ...; stop "fg" ends the request once "fg" appears,
    on the engine too (aborted, not run to max_tokens)."""
    import json as _json

    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/v1/completions", json={"prompt": [100], "max_tokens": 12, "stop": ["zz", "fg"]},
                          timeout=60).json()
        ch = r["choices"][0]
        assert ch["text"] == "de" and ch["finish_reason"] == "stop" and ch["token_ids"] == [100, 101, 102, 103]
        assert eng.aborted and eng.aborted[0][1] < 12                     # the engine stopped early
        # streamed: the text deltas add up to the cut text
        with requests.post(base + "/v1/completions", json={"prompt": [100], "max_tokens": 12, "stop": "fg",
                                                            "stream": True}, stream=True, timeout=60) as resp:
            chunks = [_json.loads(ln[6:]) for ln in resp.iter_lines(decode_unicode=True)
                      if ln.startswith("data: ") and ln != "data: [DONE]"]
        assert "".join(c["choices"][0]["text"] for c in chunks) == "de"
        assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
        # chat: same rules
        r = requests.post(base + "/v1/chat/completions",
                          json={"messages": [{"role": "user", "content": "d"}], "max_tokens": 6, "stop": "\x00"},
                          timeout=60).json()
        assert r["choices"][0]["finish_reason"] == "length"                 # no stop string in the output
        bad = requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 2, "stop": [3]}, timeout=60)
        assert bad.status_code == 400
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


class _SlowEngine(FakeEngine):
    """5 ms per step: a long request is still running when its client leaves."""

    def step(self):
        import time as _t

        _t.sleep(0.005)
        super().step()


def test_closing_a_stream_aborts_the_request():
    eng = _SlowEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    try:
        g = server.submit_stream([1, 2, 3], 1000, timeout=60)
        assert next(g)                      # the request is running
        g.close()                           # the client went away
        import time as _t
        deadline = _t.time() + 10
        while not eng.aborted and _t.time() < deadline:
            _t.sleep(0.01)
        assert eng.aborted and not eng.sched.running
        assert eng.steps < 1000                     # it did not run to max_tokens
    finally:
        server.stop()
        loop.join(timeout=30)


def _lockstep_stop(rank, world):
    import datetime

    import torch.distributed as dist

    ctrl = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, ctrl, rank, world)
    results = {}
    if rank == 0:
        def clients():
            tok = srv_mod.ByteTokenizer()
            a = threading.Thread(target=lambda: results.update(
                a=server.submit([100], 40, timeout=60, with_reason=True, stop_strs=("fg",), detok=tok.decode)))
            b = threading.Thread(target=lambda: results.update(b=server.submit([5, 6], 8, timeout=60,
                                                                              with_reason=True)))
            a.start()
            b.start()
            a.join()
            b.join()
            server.stop()

        threading.Thread(target=clients, daemon=True).start()
    server.serve_forever()
    return {"aborted": eng.aborted, "results": results, "steps": eng.steps}


def test_stop_string_abort_is_lockstep_on_two_ranks():
    res = run_ranks(_lockstep_stop, 2)
    assert res[0]["aborted"] == res[1]["aborted"] and len(res[0]["aborted"]) == 1   # same request, same step
    assert res[0]["steps"] == res[1]["steps"]
    assert res[0]["results"]["a"] == ([100, 101, 102, 103], "stop")
    assert res[0]["results"]["b"] == (expected([5, 6], 8), "length")


def test_stream_holds_back_a_possible_stop_string_then_releases_it():
    """Text that may begin a stop string is held until the next tokens
    decide: stop "fz" never completes, so "f" is sent later, not lost."""
    import json as _json

    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        for path, body, get in (
                ("/v1/completions", {"prompt": [100]}, lambda c: c["choices"][0]["text"]),
                ("/v1/chat/completions", {"messages": [{"role": "user", "content": "d"}]},
                 lambda c: c["choices"][0].get("delta", {}).get("content", ""))):
            with requests.post(base + path, json={**body, "max_tokens": 3, "stop": ["fz"], "stream": True},
                               stream=True, timeout=60) as resp:
                chunks = [_json.loads(ln[6:]) for ln in resp.iter_lines(decode_unicode=True)
                          if ln.startswith("data: ") and ln != "data: [DONE]"]
            assert chunks[-1]["choices"][0]["finish_reason"] == "length"
            if path == "/v1/completions":
                assert "".join(get(c) for c in chunks) == "def"
                assert [get(c) for c in chunks[:3]] == ["d", "e", ""]   # "f" held: it may start "fz"
            assert get(chunks[-1]) != "" or path != "/v1/completions"
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_sglang_native_generate_endpoint():
    import json as _json

    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/generate", json={"input_ids": [100], "sampling_params": {
            "max_new_tokens": 12, "stop": "fg"}}, timeout=60).json()
        assert r["text"] == "de" and r["output_ids"] == [100, 101, 102, 103]
        assert r["meta_info"] == {"prompt_tokens": 1, "completion_tokens": 4, "finish_reason": {"type": "stop"}}
        r = requests.post(base + "/generate", json={"text": "ab", "sampling_params": {"max_new_tokens": 3}},
                          timeout=60).json()
        assert r["output_ids"] == expected(list(b"ab"), 3) and r["meta_info"]["finish_reason"]["type"] == "length"
        with requests.post(base + "/generate", json={"input_ids": [5], "sampling_params": {"max_new_tokens": 4},
                                                     "stream": True}, stream=True, timeout=60) as resp:
            objs = [_json.loads(ln[6:]) for ln in resp.iter_lines(decode_unicode=True)
                    if ln.startswith("data: ") and ln != "data: [DONE]"]
        assert objs[-1]["output_ids"] == expected([5], 4) and objs[-1]["meta_info"]["finish_reason"]["type"] == "length"
        assert all(len(a["output_ids"]) <= len(b["output_ids"]) for a, b in zip(objs, objs[1:]))   # cumulative
        # chat accepts the newer max_completion_tokens spelling
        c = requests.post(base + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                               "max_completion_tokens": 2}, timeout=60).json()
        assert c["usage"]["completion_tokens"] == 2
        # a batch: one result per item, in order; per-item or shared sampling params
        rs = requests.post(base + "/generate", json={"text": ["ab", "c"], "sampling_params": [
            {"max_new_tokens": 2}, {"max_new_tokens": 3}]}, timeout=60).json()
        assert [x["output_ids"] for x in rs] == [expected(list(b"ab"), 2), expected(list(b"c"), 3)]
        rs = requests.post(base + "/generate", json={"input_ids": [[7], [8, 9]], "rid": ["a", "b"],
                                                     "sampling_params": {"max_new_tokens": 2}}, timeout=60).json()
        assert [x["output_ids"] for x in rs] == [expected([7], 2), expected([8, 9], 2)]
        assert [x["meta_info"]["id"] for x in rs] == ["a", "b"]
        for bad in ({"text": ["a", "b"], "rid": ["x"]}, {"text": ["a", "b"], "rid": ["x", "x"]},
                    {"text": ["a", "b"], "stream": True}, {"input_ids": [[1], [1] * 5000]}):
            assert requests.post(base + "/generate", json=bad, timeout=60).status_code == 400, bad
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_openai_logprobs_formats():
    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/v1/completions", json={"prompt": [100], "max_tokens": 3, "logprobs": 2},
                          timeout=60).json()
        lp = r["choices"][0]["logprobs"]
        assert lp["tokens"] == ["d", "e", "f"] and lp["token_logprobs"] == [-0.25] * 3
        assert lp["top_logprobs"][0] == {"d": -0.25, "e": -2.0} and lp["text_offset"] == [0, 1, 2]
        r = requests.post(base + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                               "max_tokens": 2, "logprobs": True, "top_logprobs": 1},
                          timeout=60).json()
        content = r["choices"][0]["logprobs"]["content"]
        assert len(content) == 2 and content[0]["logprob"] == -0.25 and len(content[0]["top_logprobs"]) == 1
        assert content[0]["bytes"] == list(content[0]["token"].encode())
        r = requests.post(base + "/v1/completions", json={"prompt": [100], "max_tokens": 2}, timeout=60).json()
        assert r["choices"][0]["logprobs"] is None
        # streamed: each chunk carries the logprobs of its own tokens
        import json as _json

        def chunks(path, body):
            with requests.post(base + path, json={**body, "stream": True}, stream=True, timeout=60) as resp:
                return [_json.loads(ln[6:]) for ln in resp.iter_lines(decode_unicode=True)
                        if ln.startswith("data: ") and ln != "data: [DONE]"]

        cs = chunks("/v1/completions", {"prompt": [100], "max_tokens": 3, "logprobs": 1})
        toks = [t for c in cs if c["choices"][0]["logprobs"] for t in c["choices"][0]["logprobs"]["tokens"]]
        assert toks == ["d", "e", "f"] and cs[-1]["choices"][0]["logprobs"] is None      # the final chunk
        assert all(c["choices"][0]["logprobs"]["top_logprobs"][0] == {t: -0.25}
                   for c, t in zip(cs, "def"))
        cs = chunks("/v1/chat/completions", {"messages": [{"role": "user", "content": "x"}], "max_tokens": 2,
                                             "logprobs": True, "top_logprobs": 2})
        items = [it for c in cs if c["choices"][0]["logprobs"] for it in c["choices"][0]["logprobs"]["content"]]
        assert len(items) == 2 and all(it["logprob"] == -0.25 and len(it["top_logprobs"]) == 2 for it in items)
        g = chunks("/generate", {"input_ids": [100], "return_logprob": True, "top_logprobs_num": 1,
                                 "sampling_params": {"max_new_tokens": 3}})
        meta = g[-1]["meta_info"]
        assert meta["output_token_logprobs"] == [[-0.25, t, None] for t in expected([100], 3)]
        assert meta["output_top_logprobs"][0] == [[-0.25, 100, None]]
        assert requests.post(base + "/generate", json={"input_ids": [100], "return_logprob": True,
                                                       "logprob_start_len": 0, "stream": True},
                             timeout=60).status_code == 400
        assert "usage" in chunks("/v1/completions", {"prompt": [100], "max_tokens": 2})[-1]
        for path, body in (("/v1/completions", {"prompt": [100], "max_tokens": 2}),
                           ("/v1/chat/completions", {"messages": [{"role": "user", "content": "x"}],
                                                     "max_tokens": 2})):
            assert all("usage" not in c for c in chunks(path, {**body, "stream_options": {"include_usage": False}}))
        plain = chunks("/v1/completions", {"prompt": [100], "max_tokens": 2})
        assert all(c["choices"][0]["logprobs"] is None for c in plain)
        assert requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 2, "echo": True,
                                                             "stream": True}, timeout=60).status_code == 400
        # with a stop string the logprobs are cut with the tokens
        r = requests.post(base + "/v1/completions", json={"prompt": [100], "max_tokens": 9, "logprobs": 0,
                                                          "stop": "fg"}, timeout=60).json()
        assert len(r["choices"][0]["logprobs"]["tokens"]) == len(r["choices"][0]["token_ids"]) == 4
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_echo_scores_the_prompt():
    """``echo`` with ``logprobs``: the prompt's tokens and logprobs come first
    (None for the first token); ``max_tokens`` 0 scores without generating.
    sglang's /generate returns the same through ``return_logprob``."""
    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/v1/completions", json={"prompt": [97, 98, 99], "max_tokens": 0, "echo": True,
                                                          "logprobs": 0}, timeout=60).json()
        ch = r["choices"][0]
        assert ch["text"] == "abc" and ch["token_ids"] == []
        assert ch["logprobs"]["tokens"] == ["a", "b", "c"] and ch["logprobs"]["token_logprobs"] == [None, -1.0, -1.0]
        assert ch["logprobs"]["top_logprobs"][0] is None
        r = requests.post(base + "/v1/completions", json={"prompt": [97, 98], "max_tokens": 2, "echo": True,
                                                          "logprobs": 1}, timeout=60).json()
        lp = r["choices"][0]["logprobs"]
        assert lp["tokens"][:2] == ["a", "b"] and len(lp["tokens"]) == 4
        assert lp["token_logprobs"] == [None, -1.0, -0.25, -0.25]
        assert r["choices"][0]["text"].startswith("ab")
        g = requests.post(base + "/generate", json={"input_ids": [97, 98, 99], "sampling_params": {
            "max_new_tokens": 2}, "return_logprob": True, "logprob_start_len": 0, "top_logprobs_num": 1},
            timeout=60).json()
        m = g["meta_info"]
        assert m["input_token_logprobs"] == [[None, 97, None], [-1.0, 98, None], [-1.0, 99, None]]
        assert [x[1] for x in m["output_token_logprobs"]] == g["output_ids"] and len(m["output_top_logprobs"]) == 2
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_n_choices_per_request():
    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/v1/completions", json={"prompt": [7, 8], "max_tokens": 3, "n": 3,
                                                          "temperature": 0.9, "seed": 40}, timeout=60).json()
        assert [c["index"] for c in r["choices"]] == [0, 1, 2] and r["usage"]["completion_tokens"] == 9
        assert sorted(s_.seed for s_ in eng.sampling_seen[-3:]) == [40, 41, 42]   # choice i draws with seed + i
        c = requests.post(base + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                               "max_tokens": 2, "n": 2}, timeout=60).json()
        assert len(c["choices"]) == 2 and c["usage"]["completion_tokens"] == 4
        bad = requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 2, "n": 2, "stream": True},
                            timeout=60)
        assert bad.status_code == 400
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_serving_bench_against_the_server():
    """benchmarks/bench_serving.py: streamed requests under a concurrency cap
    and a Poisson arrival rate, timed by the client."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_serving", os.path.join(ROOT, "benchmarks", "bench_serving.py"))
    bs = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bs)
    eng = _SlowEngine()
    server, loop, http, base = _serve(eng)
    try:
        res = bs.main(["--url", base, "--num-requests", "12", "--concurrency", "4", "--request-rate", "50",
                       "--input-len", "5:20", "--output-len", "6"])
        assert res["completed"] == 12 and res["errors"] == 0
        assert res["output_tok_s"] > 0 and res["ttft_ms"]["p50"] > 0 and res["itl_ms"]["p50"] > 0
        assert res["latency_ms"]["p99"] >= res["latency_ms"]["p50"] >= res["ttft_ms"]["p50"]
        assert len(eng.log) == 12 and all(m == 6 for _, _, m in eng.log)
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_example_client_against_the_server(capsys):
    import importlib.util

    spec = importlib.util.spec_from_file_location("client", os.path.join(ROOT, "examples", "client.py"))
    client = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(client)
    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        client.main(["--url", base, "--prompt", "hi", "--max-tokens", "4"])
        client.main(["--url", base, "--prompt", "hi", "--max-tokens", "4", "--stream"])
        out = capsys.readouterr().out
        assert "tok/s" in out and "prompt=" in out
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_api_key_guards_the_model_endpoints():
    import requests

    from conftest import free_port

    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "served-name", api_key="s3cret"), "127.0.0.1", port)
    base = f"http://127.0.0.1:{port}"
    try:
        body = {"prompt": [1, 2], "max_tokens": 2}
        assert requests.post(base + "/v1/completions", json=body, timeout=30).status_code == 401
        assert requests.post(base + "/v1/completions", json=body, timeout=30,
                             headers={"Authorization": "Bearer wrong"}).status_code == 401
        ok = requests.post(base + "/v1/completions", json=body, timeout=30, headers={"Authorization": "Bearer s3cret"})
        assert ok.status_code == 200 and ok.json()["model"] == "served-name"
        assert requests.get(base + "/health", timeout=30).status_code == 200      # probes stay open
        assert requests.get(base + "/v1/models", timeout=30).status_code == 401
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_health_reports_a_communicator_error():
    import requests

    class _Comm:
        code = 0

        def err(self):
            return self.code

        counters = {}

    eng = FakeEngine()
    comm = _Comm()
    eng.tp = type("TP", (), {"ca_comm": comm})()
    server, loop, http, base = _serve(eng)
    try:
        assert requests.get(base + "/health", timeout=30).status_code == 200
        comm.code = 3                                   # a device wait timed out
        h = requests.get(base + "/health", timeout=30)
        assert h.status_code == 503 and h.json()["communicator_error"] == 3
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_several_prompts_in_one_completion_request():
    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/v1/completions", json={"prompt": [[1, 2], [10], "a"], "max_tokens": 2, "n": 2},
                          timeout=60).json()
        got = [c["token_ids"] for c in r["choices"]]
        want = [expected(p, 2) for p in ([1, 2], [1, 2], [10], [10], [97], [97])]
        assert got == want and [c["index"] for c in r["choices"]] == list(range(6))
        assert r["usage"]["prompt_tokens"] == (2 + 1 + 1) * 2 and r["usage"]["completion_tokens"] == 12
        # lm-eval style scoring of several texts at once
        r = requests.post(base + "/v1/completions", json={"prompt": ["ab", "cd"], "max_tokens": 0, "echo": True,
                                                          "logprobs": 0}, timeout=60).json()
        assert [c["text"] for c in r["choices"]] == ["ab", "cd"]
        assert [c["logprobs"]["token_logprobs"] for c in r["choices"]] == [[None, -1.0], [None, -1.0]]
        bad = requests.post(base + "/v1/completions", json={"prompt": [[1], [2] * 5000], "max_tokens": 2},
                            timeout=60)
        assert bad.status_code == 400
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_chat_template_override():
    import requests

    from conftest import free_port

    tpl = "{% for m in messages %}[{{ m.role }}]{{ m.content }}{% endfor %}{% if add_generation_prompt %}>{% endif %}"
    tok = srv_mod.ByteTokenizer(srv_mod.load_chat_template(tpl))
    assert tok.chat([{"role": "user", "content": "hi"}]) == list(b"[user]hi>")
    assert srv_mod.ByteTokenizer().chat([{"role": "user", "content": "x"}]) == list(b"<|user|>x<|assistant|>")
    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake", tok), "127.0.0.1", port)
    try:
        requests.post(f"http://127.0.0.1:{port}/v1/chat/completions",
                      json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 1}, timeout=30)
        assert eng.log[-1][1] == tuple(b"[user]hi>")
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_server_entry_point_end_to_end_on_cpu():
    """``python -m <pkg>.server --tp 2`` for real: the launcher starts two
    ranks under torch.distributed.run, each builds the oracle engine on CPU
    (gloo collectives), rank 0 serves HTTP; SIGTERM stops every rank."""
    import signal as _signal
    import time as _t

    import requests

    from conftest import free_port

    port = free_port()
    env = dict(os.environ)
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK", "MASTER_PORT"):
        env.pop(k, None)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    cmd = [sys.executable, "-m", "3080_mod_p2p_sglang_patch_b200.server", "--model", "tiny", "--impl", "oracle",
           "--device", "cpu", "--tp", "2", "--port", str(port), "--max-batch", "4", "--max-seq", "512",
           "--chunk", "64"]
    proc = subprocess.Popen(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                            start_new_session=True)
    base = f"http://127.0.0.1:{port}"
    try:
        deadline = _t.time() + 240
        while _t.time() < deadline:
            try:
                if requests.get(base + "/health", timeout=2).status_code == 200:
                    break
            except requests.ConnectionError:
                pass
            assert proc.poll() is None, proc.stdout.read().decode()[-3000:]
            _t.sleep(0.5)
        r = requests.post(base + "/v1/completions", json={"prompt": "hello", "max_tokens": 4}, timeout=120)
        assert r.status_code == 200 and len(r.json()["choices"][0]["token_ids"]) == 4
        c = requests.post(base + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                               "max_tokens": 3, "temperature": 0.7, "seed": 1},
                          timeout=120)
        assert c.status_code == 200 and c.json()["usage"]["completion_tokens"] == 3
        proc.send_signal(_signal.SIGTERM)
        proc.wait(timeout=90)
    finally:
        if proc.poll() is None:
            os.killpg(proc.pid, _signal.SIGKILL)   # the process group this test started
            proc.wait(timeout=30)


def test_sampling_adjustments_reach_the_engine():
    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        r = requests.post(base + "/v1/completions", json={
            "prompt": [1, 2], "max_tokens": 2, "presence_penalty": 0.5, "frequency_penalty": 0.25,
            "repetition_penalty": 1.1, "logit_bias": {"7": 5, "3": -100}, "min_tokens": 2}, timeout=30)
        assert r.status_code == 200
        sp = eng.sampling_seen[-1]
        assert (sp.temperature, sp.presence_penalty, sp.frequency_penalty, sp.repetition_penalty) == (0.0, 0.5, 0.25, 1.1)
        assert sp.logit_bias == ((3, -100.0), (7, 5.0)) and sp.min_new_tokens == 2
        requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 1}, timeout=30)
        assert eng.sampling_seen[-1] is None                                # plain greedy: no adjustments
        bad = requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 1,
                                                            "logit_bias": {"x": 1}}, timeout=30)
        assert bad.status_code == 400
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_request_log_lines(caplog):
    import json as _json
    import logging

    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096, log_requests=True)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    try:
        with caplog.at_level(logging.INFO, logger=srv_mod.__name__):
            server.submit([1, 2, 3], 4, timeout=30)
        lines = [r.getMessage() for r in caplog.records if r.getMessage().startswith("request ")]
        rec = _json.loads(lines[-1][len("request "):])
        assert rec["prompt_tokens"] == 3 and rec["output_tokens"] == 4 and rec["finish_reason"] == "length"
        assert rec["e2e_ms"] >= rec["ttft_ms"] >= 0
    finally:
        server.stop()
        loop.join(timeout=30)


def test_more_sglang_launch_flags_parse():
    p = srv_mod.build_parser()
    a = p.parse_args(["--model", "tiny", "--dtype", "bfloat16", "--kv-cache-dtype", "auto", "--quantization", "awq",
                      "--random-seed", "7", "--log-level", "warning", "--max-total-tokens", "100000",
                      "--disable-radix-cache", "--log-requests"])
    assert (a.quantization, a.seed, a.log_level, a.max_total_tokens, a.disable_radix_cache, a.log_requests) == \
        ("awq", 7, "warning", 100000, True, True)
    import pytest as _pt
    with _pt.raises(SystemExit):
        p.parse_args(["--kv-cache-dtype", "fp8_e5m2"])      # not supported: refused, not ignored
    g = p.parse_args(["--cuda-graph-bs", "1", "4", "16", "--cuda-graph-max-bs", "12"])
    assert g.cuda_graph_bs == [1, 4, 16] and g.cuda_graph_max_bs == 12
    c = p.parse_args(["--disable-custom-all-reduce", "--trust-remote-code"])
    assert c.disable_custom_all_reduce and c.trust_remote_code
    assert not p.parse_args([]).disable_custom_all_reduce


def test_overload_bound_refuses_with_503_and_recovers():
    import requests

    from conftest import free_port

    eng = _SlowEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096, max_queued=2)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    url = f"http://127.0.0.1:{port}/v1/completions"
    try:
        results = []
        ths = [threading.Thread(target=lambda: results.append(
            requests.post(url, json={"prompt": [1], "max_tokens": 60}, timeout=60).status_code)) for _ in range(2)]
        for t in ths:
            t.start()
        import time as _t
        deadline = _t.time() + 10
        while server._live < 2 and _t.time() < deadline:
            _t.sleep(0.01)
        r = requests.post(url, json={"prompt": [2], "max_tokens": 2}, timeout=60)
        assert r.status_code == 503                                   # two in flight: refused
        s = requests.post(url, json={"prompt": [2], "max_tokens": 2, "stream": True}, timeout=60)
        assert s.status_code == 503                                   # a stream is refused up front too
        for t in ths:
            t.join()
        assert results == [200, 200] and server._live == 0
        assert requests.post(url, json={"prompt": [3], "max_tokens": 2}, timeout=60).status_code == 200
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_admin_endpoints():
    import requests

    eng = FakeEngine()
    server, loop, http, base = _serve(eng)
    try:
        assert requests.post(base + "/tokenize", json={"text": "hi"}, timeout=30).json() == {"tokens": [104, 105]}
        assert requests.post(base + "/detokenize", json={"tokens": [104, 105]}, timeout=30).json() == {"text": "hi"}
        assert requests.get(base + "/get_model_info", timeout=30).json()["model_path"] == "fake"
        assert requests.get(base + "/get_server_info", timeout=30).json()["tp_size"] == 1
        assert requests.post(base + "/flush_cache", timeout=30).json() == {"status": "ok"}
        r = requests.post(base + "/v1/completions", json={"prompt": [1], "max_tokens": 2}, timeout=30)
        assert r.status_code == 200                                             # still serving after the flush
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_abort_by_request_id_and_health_generate():
    """sglang's ``rid`` on /generate and /abort_request: the named request ends
    early with finish reason "abort"; a second request with a live id is
    refused; unknown ids report aborted=False; /health_generate steps the loop."""
    import time as _t

    import requests

    eng = _SlowEngine()
    server, loop, http, base = _serve(eng)
    try:
        assert requests.get(base + "/health_generate", timeout=60).json() == {"status": "ok"}
        res = []
        th = threading.Thread(target=lambda: res.append(requests.post(
            base + "/generate", json={"input_ids": [1, 2], "rid": "job-7",
                                      "sampling_params": {"max_new_tokens": 1000}}, timeout=60).json()))
        th.start()
        deadline = _t.time() + 10
        while "job-7" not in server._named and _t.time() < deadline:
            _t.sleep(0.01)
        dup = requests.post(base + "/generate", json={"input_ids": [1], "rid": "job-7",
                                                      "sampling_params": {"max_new_tokens": 2}}, timeout=60)
        assert dup.status_code == 400                                   # the id is in flight
        assert requests.post(base + "/abort_request", json={"rid": "nope"}, timeout=30).json()["aborted"] is False
        assert requests.post(base + "/abort_request", json={"rid": "job-7"}, timeout=30).json()["aborted"] is True
        th.join(timeout=30)
        meta = res[0]["meta_info"]
        assert meta["finish_reason"]["type"] == "abort" and meta["id"] == "job-7"
        assert meta["completion_tokens"] < 1000
        assert "job-7" not in server._named and server._live == 0
        ok = requests.post(base + "/generate", json={"input_ids": [1], "rid": "job-7",
                                                     "sampling_params": {"max_new_tokens": 2}}, timeout=60)
        assert ok.status_code == 200                                    # the id is free again
        assert requests.post(base + "/abort_request", json={}, timeout=30).status_code == 400
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_metrics_gauges_on_the_oracle_engine():
    """Queue, running and KV-cache gauges read the real scheduler and page
    allocator: pages held by the prefix cache after a request count as used."""
    import requests

    from conftest import free_port

    eng_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine")
    models = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models")
    eng = eng_mod.LLMEngine(models.LlamaConfig.tiny(), impl="oracle", device="cpu", max_batch=2, max_seq=256,
                            chunk=64, use_graphs=False, prefix_cache=True)
    server = srv_mod.EngineServer(eng, max_prompt=eng.max_seq)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "tiny"), "127.0.0.1", port)
    base = f"http://127.0.0.1:{port}"
    try:
        def gauges():
            return {ln.split()[0]: float(ln.split()[1]) for ln in requests.get(base + "/metrics", timeout=30)
                    .text.splitlines() if ln.startswith(("mbx_num_", "mbx_kv_", "mbx_requests_in_flight"))}

        g0 = gauges()
        assert g0 == {"mbx_requests_in_flight": 0, "mbx_num_queue_reqs": 0, "mbx_num_prefill_reqs": 0,
                      "mbx_num_running_reqs": 0, "mbx_kv_cache_usage": 0}
        r = requests.post(base + "/v1/completions", json={"prompt": list(range(1, 40)), "max_tokens": 2}, timeout=120)
        assert r.status_code == 200
        g1 = gauges()
        assert g1["mbx_num_running_reqs"] == 0 and g1["mbx_requests_in_flight"] == 0
        assert 0 < g1["mbx_kv_cache_usage"] <= 1            # the prompt's full pages stay in the prefix cache
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True


def test_ignore_eos_overrides_the_default_stop_ids():
    import requests

    from conftest import free_port

    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096, stop_ids=(101,))    # the "EOS" is token 101
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    base = f"http://127.0.0.1:{port}"
    try:
        body = {"prompt": [100], "max_tokens": 4}
        r = requests.post(base + "/v1/completions", json=body, timeout=60).json()["choices"][0]
        assert r["token_ids"] == [100, 101] and r["finish_reason"] == "stop"
        r = requests.post(base + "/v1/completions", json={**body, "ignore_eos": True}, timeout=60).json()
        assert r["choices"][0]["token_ids"] == expected([100], 4)
        g = requests.post(base + "/generate", json={"input_ids": [100], "sampling_params": {
            "max_new_tokens": 4, "ignore_eos": True}}, timeout=60).json()
        assert g["output_ids"] == expected([100], 4) and g["meta_info"]["finish_reason"]["type"] == "length"
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True
