"""Data-parallel router (``router.py``, ``server --dp N``) over in-process
servers on CPU: least-in-flight routing, pass-through of plain and streamed
responses, health and metrics of every replica, failover when a replica is
down, and the replica launch commands (GPU partition, ports)."""
import importlib
import json
import threading
import time

import pytest
import requests

from conftest import free_port
from test_server_cpu import FakeEngine, expected

srv_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.server")
rt_mod = importlib.import_module("3080_mod_p2p_sglang_patch_b200.router")


def _replica():
    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake"), "127.0.0.1", port)
    return {"eng": eng, "server": server, "loop": loop, "http": http, "url": f"http://127.0.0.1:{port}"}


def _stop(rep):
    rep["server"].stop()
    rep["loop"].join(timeout=30)
    rep["http"].should_exit = True


def test_order_prefers_the_least_loaded_replica_and_rotates_ties():
    r = rt_mod.Router(["http://a", "http://b", "http://c"])
    firsts = {r.order()[0] for _ in range(6)}
    assert firsts == {0, 1, 2}                      # ties rotate
    r.inflight = [3, 0, 1]
    assert r.order() == [1, 2, 0]


def test_router_over_two_replicas():
    reps = [_replica(), _replica()]
    router = rt_mod.Router([rp["url"] for rp in reps])
    port = free_port()
    http, _ = srv_mod.start_http(rt_mod.build_router_app(router), "127.0.0.1", port)
    base = f"http://127.0.0.1:{port}"
    try:
        results = {}

        def one(i):
            r = requests.post(base + "/v1/completions", json={"prompt": [i, i + 1], "max_tokens": 3}, timeout=60)
            results[i] = r.json()["choices"][0]["token_ids"]

        ths = [threading.Thread(target=one, args=(i,)) for i in range(8)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        assert all(results[i] == expected([i, i + 1], 3) for i in range(8))
        assert sum(router.routed) == 8 and min(router.routed) > 0        # both replicas served
        assert len(reps[0]["eng"].log) + len(reps[1]["eng"].log) == 8
        # streaming passes through
        with requests.post(base + "/v1/completions", json={"prompt": [4, 5], "max_tokens": 4, "stream": True},
                           stream=True, timeout=60) as r:
            lines = [ln for ln in r.iter_lines(decode_unicode=True) if ln.startswith("data: ")]
        assert lines[-1] == "data: [DONE]"
        toks = sum((json.loads(ln[6:])["choices"][0]["token_ids"] for ln in lines[:-1]), [])
        assert toks == expected([4, 5], 4)
        h = requests.get(base + "/health", timeout=30).json()
        assert h["status"] == "ok" and len(h["replicas"]) == 2
        m = requests.get(base + "/metrics", timeout=30).text
        assert 'mbx_requests_total{replica="0"}' in m and 'mbx_requests_total{replica="1"}' in m
        assert 'mbx_router_requests_total{replica="1"}' in m
        assert requests.get(base + "/v1/models", timeout=30).json()["data"][0]["id"] == "fake"
        g = requests.post(base + "/generate", json={"input_ids": [3], "sampling_params": {"max_new_tokens": 2}},
                          timeout=60).json()
        assert g["output_ids"] == expected([3], 2)
        assert requests.post(base + "/flush_cache", timeout=30).json()["status"] == "ok"
        assert requests.post(base + "/tokenize", json={"text": "a"}, timeout=30).json() == {"tokens": [97]}
        assert requests.get(base + "/get_model_info", timeout=30).json()["model_path"] == "fake"
        assert requests.get(base + "/health_generate", timeout=60).json()["status"] == "ok"
        assert requests.post(base + "/abort_request", json={"rid": "none"}, timeout=30).json()["aborted"] is False
        # one replica goes down: requests fail over to the other
        _stop(reps[1])
        time.sleep(0.5)
        for i in range(4):
            r = requests.post(base + "/v1/completions", json={"prompt": [7, i], "max_tokens": 2}, timeout=60)
            assert r.status_code == 200 and r.json()["choices"][0]["token_ids"] == expected([7, i], 2)
        assert requests.get(base + "/health", timeout=30).status_code == 503
    finally:
        http.should_exit = True
        _stop(reps[0])
        if reps[1]["loop"].is_alive():
            _stop(reps[1])


def test_replica_commands_partition_gpus_and_ports():
    cmds = srv_mod.replica_commands(["--model", "tiny", "--tp", "2", "--dp", "2", "--port", "9000"], 2, 2, 9000,
                                    ["4", "5", "6", "7"])
    assert [env["CUDA_VISIBLE_DEVICES"] for env, _ in cmds] == ["4,5", "6,7"]
    for i, (_, cmd) in enumerate(cmds):
        assert "torch.distributed.run" in cmd and "--nproc-per-node=2" in cmd
        assert cmd[-2:] == ["--port", str(9001 + i)] and "--dp" not in cmd and "--tp" not in cmd
    single = srv_mod.replica_commands(["--model", "tiny", "--dp=2"], 1, 2, 8001)
    assert [env["CUDA_VISIBLE_DEVICES"] for env, _ in single] == ["0", "1"]
    assert all("torch.distributed.run" not in cmd for _, cmd in single)
    with pytest.raises(SystemExit):
        srv_mod.replica_commands([], 2, 4, 8001, ["0", "1", "2"])


def test_router_passes_the_api_key_to_replicas():
    eng = FakeEngine()
    server = srv_mod.EngineServer(eng, max_prompt=4096)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    rep_http, _ = srv_mod.start_http(srv_mod.build_app(server, "fake", api_key="k1"), "127.0.0.1", port)
    router = rt_mod.Router([f"http://127.0.0.1:{port}"])
    rport = free_port()
    http, _ = srv_mod.start_http(rt_mod.build_router_app(router), "127.0.0.1", rport)
    base = f"http://127.0.0.1:{rport}"
    try:
        body = {"prompt": [3, 4], "max_tokens": 2}
        assert requests.post(base + "/v1/completions", json=body, timeout=30).status_code == 401
        r = requests.post(base + "/v1/completions", json=body, headers={"Authorization": "Bearer k1"}, timeout=30)
        assert r.status_code == 200 and r.json()["choices"][0]["token_ids"] == expected([3, 4], 2)
        with requests.post(base + "/v1/completions", json={**body, "stream": True}, stream=True, timeout=30,
                           headers={"Authorization": "Bearer k1"}) as s:
            assert any(ln == "data: [DONE]" for ln in s.iter_lines(decode_unicode=True))
        assert requests.get(base + "/v1/models", headers={"Authorization": "Bearer k1"}, timeout=30).status_code == 200
    finally:
        http.should_exit = True
        rep_http.should_exit = True
        server.stop()
        loop.join(timeout=30)


def test_dp_entry_point_end_to_end_on_cpu():
    """``server --dp 2`` for real: two oracle replicas on CPU behind the router."""
    import os
    import signal as _signal
    import subprocess
    import sys

    port = free_port()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK", "MASTER_PORT"):
        env.pop(k, None)
    env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
    cmd = [sys.executable, "-m", "3080_mod_p2p_sglang_patch_b200.server", "--model", "tiny", "--impl", "oracle",
           "--device", "cpu", "--dp", "2", "--port", str(port), "--max-batch", "4", "--max-seq", "512"]
    proc = subprocess.Popen(cmd, env=env, cwd=root, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                            start_new_session=True)
    base = f"http://127.0.0.1:{port}"
    try:
        deadline = time.time() + 240
        while time.time() < deadline:
            try:
                if requests.get(base + "/health", timeout=2).status_code == 200:
                    break
            except requests.ConnectionError:
                pass
            assert proc.poll() is None, proc.stdout.read().decode()[-3000:]
            time.sleep(0.5)
        outs = []
        for i in range(4):
            r = requests.post(base + "/v1/completions", json={"prompt": [5 + i, 6], "max_tokens": 3}, timeout=120)
            assert r.status_code == 200
            outs.append(r.json()["choices"][0]["token_ids"])
        m = requests.get(base + "/metrics", timeout=30).text
        assert 'mbx_router_requests_total{replica="0"}' in m and 'mbx_router_requests_total{replica="1"}' in m
        assert all(len(o) == 3 for o in outs)
        proc.send_signal(_signal.SIGTERM)
        proc.wait(timeout=90)
    finally:
        if proc.poll() is None:
            os.killpg(proc.pid, _signal.SIGKILL)   # the process group this test started
            proc.wait(timeout=30)
