"""Data-parallel front end: one OpenAI-compatible endpoint over N server
replicas, each an independent TP group on its own GPUs (the role of sglang's
``--dp-size`` data-parallel controller; the reference runs one TP=2 group).

    python -m 3080_mod_p2p_sglang_patch_b200.router --backends http://127.0.0.1:8101,http://127.0.0.1:8102 --port 8001

``server --dp N`` starts the replicas and this router together. Each request
goes to the replica with the fewest requests in flight (ties: round robin),
streamed responses pass through as they arrive, and a replica that refuses
the connection is skipped for that request. ``/health`` reports every
replica, ``/metrics`` concatenates the replicas' metrics with a ``replica``
label plus the router's own counters.
"""
import argparse
import itertools
import json
import logging
import threading

logger = logging.getLogger(__name__)


class Router:
    def __init__(self, backends, timeout: float = 600.0):
        if not backends:
            raise ValueError("no backends")
        self.backends = [b.rstrip("/") for b in backends]
        self.timeout = timeout
        self.inflight = [0] * len(self.backends)
        self.routed = [0] * len(self.backends)
        self.failed = [0] * len(self.backends)
        self._lock = threading.Lock()
        self._rr = itertools.count()

    def order(self):
        """Replica indices to try: fewest in flight first, ties rotated."""
        with self._lock:
            start = next(self._rr) % len(self.backends)
            idx = [(start + i) % len(self.backends) for i in range(len(self.backends))]
            return sorted(idx, key=lambda i: self.inflight[i])

    def _acquire(self, i):
        with self._lock:
            self.inflight[i] += 1
            self.routed[i] += 1

    def _release(self, i):
        with self._lock:
            self.inflight[i] -= 1

    def post(self, path: str, body: dict, headers: dict = None):
        """Forward a non-streaming request: (status, json body, replica)."""
        import requests

        last = None
        for i in self.order():
            self._acquire(i)
            try:
                r = requests.post(self.backends[i] + path, json=body, timeout=self.timeout, headers=headers)
                return r.status_code, r.json(), i
            except requests.ConnectionError as e:  # replica down: try the next one
                with self._lock:
                    self.failed[i] += 1
                last = e
            finally:
                self._release(i)
        raise ConnectionError(f"no replica reachable ({last})")

    def stream(self, path: str, body: dict, headers: dict = None):
        """Forward a streaming request; yields the replica's server-sent-event
        lines (each ending in a blank line) as they arrive."""
        import requests

        last = None
        for i in self.order():
            self._acquire(i)
            try:
                try:
                    r = requests.post(self.backends[i] + path, json=body, timeout=self.timeout, stream=True,
                                      headers=headers)
                except requests.ConnectionError as e:
                    with self._lock:
                        self.failed[i] += 1
                    last = e
                    continue
                with r:
                    for line in r.iter_lines(decode_unicode=True):
                        if line:
                            yield line + "\n\n"
                return
            finally:
                self._release(i)
        yield "data: " + json.dumps({"error": {"message": f"no replica reachable ({last})"}}) + "\n\n"
        yield "data: [DONE]\n\n"

    def get(self, i: int, path: str, headers: dict = None):
        import requests

        return requests.get(self.backends[i] + path, timeout=30, headers=headers)


def _relabel(text: str, replica: int) -> list:
    """Prometheus sample lines of one replica with a replica="i" label added."""
    out = []
    for line in text.splitlines():
        if not line or line.startswith("#"):
            continue
        name, _, value = line.rpartition(" ")
        if "{" in name:
            name = name[:-1] + f',replica="{replica}"}}'
        else:
            name = name + f'{{replica="{replica}"}}'
        out.append(f"{name} {value}")
    return out


def build_router_app(router: Router):
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.concurrency import iterate_in_threadpool, run_in_threadpool
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI()

    def _auth(request):
        """The client's credentials travel to the replica, which checks them."""
        a = request.headers.get("authorization")
        return {"Authorization": a} if a else None

    async def forward(path, body, request):
        if body.get("stream"):
            return StreamingResponse(iterate_in_threadpool(router.stream(path, body, _auth(request))),
                                     media_type="text/event-stream")
        try:
            status, data, _ = await run_in_threadpool(router.post, path, body, _auth(request))
        except ConnectionError as e:
            raise HTTPException(503, str(e)) from e
        return JSONResponse(data, status_code=status)

    @app.post("/v1/completions")
    async def completions(body: dict, request: Request):
        return await forward("/v1/completions", body, request)

    @app.post("/v1/chat/completions")
    async def chat(body: dict, request: Request):
        return await forward("/v1/chat/completions", body, request)

    @app.post("/generate")
    async def generate(body: dict, request: Request):
        return await forward("/generate", body, request)

    @app.post("/flush_cache")
    def flush_cache(request: Request):
        """Every replica drops its unreferenced prefix pages."""
        import requests

        out = []
        for i, b in enumerate(router.backends):
            try:
                r = requests.post(b + "/flush_cache", timeout=30, headers=_auth(request))
                out.append({"url": b, "status_code": r.status_code})
            except requests.ConnectionError as e:
                out.append({"url": b, "error": str(e)})
        ok = all(x.get("status_code") == 200 for x in out)
        return JSONResponse({"status": "ok" if ok else "partial", "replicas": out}, status_code=200 if ok else 503)

    @app.post("/abort_request")
    def abort_request(body: dict, request: Request):
        """Sent to every replica: only the one running the request knows its id."""
        import requests

        aborted = False
        for b in router.backends:
            try:
                r = requests.post(b + "/abort_request", json=body, timeout=30, headers=_auth(request))
                if r.status_code == 400:
                    return JSONResponse(r.json(), status_code=400)
                aborted = aborted or bool(r.status_code == 200 and r.json().get("aborted"))
            except requests.ConnectionError:
                continue
        return {"rid": body.get("rid"), "aborted": aborted}

    @app.get("/health_generate")
    def health_generate():
        """One generated token on every replica."""
        reps = []
        for i, b in enumerate(router.backends):
            try:
                reps.append({"url": b, **router.get(i, "/health_generate").json()})
            except Exception as e:  # noqa: BLE001
                reps.append({"url": b, "status": "down", "error": str(e)})
        ok = all(r.get("status") == "ok" for r in reps)
        return JSONResponse({"status": "ok" if ok else "degraded", "replicas": reps}, status_code=200 if ok else 503)

    def _any(method, path, request, body=None):
        """A read-only call answered by the first replica that answers."""
        import requests

        for b in router.backends:
            try:
                r = requests.request(method, b + path, json=body, timeout=30, headers=_auth(request))
                return JSONResponse(r.json(), status_code=r.status_code)
            except requests.ConnectionError:
                continue
        raise HTTPException(503, "no replica reachable")

    @app.get("/get_model_info")
    def model_info(request: Request):
        return _any("GET", "/get_model_info", request)

    @app.get("/get_server_info")
    def server_info(request: Request):
        return _any("GET", "/get_server_info", request)

    @app.post("/tokenize")
    def tokenize(body: dict, request: Request):
        return _any("POST", "/tokenize", request, body)

    @app.post("/detokenize")
    def detokenize(body: dict, request: Request):
        return _any("POST", "/detokenize", request, body)

    @app.get("/v1/models")
    def models(request: Request):
        for i in range(len(router.backends)):
            try:
                r = router.get(i, "/v1/models", _auth(request))
                return JSONResponse(r.json(), status_code=r.status_code)
            except Exception:  # noqa: BLE001 - try the next replica
                continue
        raise HTTPException(503, "no replica reachable")

    @app.get("/health")
    def health():
        reps = []
        for i, b in enumerate(router.backends):
            try:
                reps.append({"url": b, **router.get(i, "/health").json()})
            except Exception as e:  # noqa: BLE001
                reps.append({"url": b, "status": "down", "error": str(e)})
        ok = all(r.get("status") == "ok" for r in reps)
        return JSONResponse({"status": "ok" if ok else "degraded", "replicas": reps}, status_code=200 if ok else 503)

    @app.get("/metrics")
    def metrics():
        lines = ["# HELP mbx_router_requests_total Requests routed to each replica.",
                 "# TYPE mbx_router_requests_total counter"]
        lines += [f'mbx_router_requests_total{{replica="{i}"}} {n}' for i, n in enumerate(router.routed)]
        lines += ["# HELP mbx_router_inflight Requests in flight per replica.", "# TYPE mbx_router_inflight gauge"]
        lines += [f'mbx_router_inflight{{replica="{i}"}} {n}' for i, n in enumerate(router.inflight)]
        lines += ["# HELP mbx_router_connect_failures_total Refused connections per replica.",
                  "# TYPE mbx_router_connect_failures_total counter"]
        lines += [f'mbx_router_connect_failures_total{{replica="{i}"}} {n}' for i, n in enumerate(router.failed)]
        for i in range(len(router.backends)):
            try:
                lines += _relabel(router.get(i, "/metrics").text, i)
            except Exception:  # noqa: BLE001 - a down replica has no metrics
                continue
        return PlainTextResponse("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    return app


def main(argv=None):
    from .server import start_http

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--backends", required=True, help="comma-separated replica base URLs")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8001)
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(name)s %(message)s")
    router = Router(args.backends.split(","))
    srv, th = start_http(build_router_app(router), args.host, args.port)
    logger.info("routing http://%s:%d over %d replicas", args.host, args.port, len(router.backends))
    try:
        th.join()
    except KeyboardInterrupt:
        srv.should_exit = True


if __name__ == "__main__":
    main()
