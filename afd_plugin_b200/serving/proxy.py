"""Load-balancing proxy in front of completion servers, with prefill -> decode disaggregation.

Two modes, the ones of the reference's proxy tool (``tools/proxy_server.py``):

* ``--backends``: each ``POST /v1/completions`` (or ``/v1/chat/completions``)
  goes to the backend with the least load in flight (ties: round robin) and
  the answer is forwarded.
* ``--prefill`` + ``--decode``: the request first runs on a prefill server with
  ``max_tokens=1`` and ``kv_transfer_params={"do_remote_decode": true}``
  (the prefill leg of ``tools/proxy_server.py:850-867``); that server keeps the
  request's cache rows and answers with where to fetch them.  The original
  request then goes to a decode server with those ``kv_transfer_params``; it
  pulls the rows and decodes.  If the decode leg fails, the proxy asks the
  prefill server to drop the held rows.

Load is counted in prompt tokens for prefill servers and in requested tokens
for decode servers, so long prompts spread over the prefill pool the way the
reference's length-based scores do (``tools/proxy_server.py:205-211``).
Streaming requests (``"stream": true``) are relayed chunk by chunk; in the
disaggregated mode only the decode leg streams.  ``GET /health`` (alias
``/healthcheck``) reports every backend; ``POST /instances/add`` and
``/instances/remove`` change the pools while serving; ``POST
/reset_prefix_cache`` is forwarded to every backend.

    python -m afd_plugin_b200.serving.proxy --backends http://127.0.0.1:8001,http://127.0.0.1:8002 --port 8000
    python -m afd_plugin_b200.serving.proxy --prefill http://127.0.0.1:8001 --decode http://127.0.0.1:8002
"""

from __future__ import annotations

import argparse
import threading

import requests
from fastapi import Request


def normalize_url(addr: str) -> str:
    """``host:port`` or a URL -> ``http://host:port`` without a trailing slash."""
    addr = addr.strip().rstrip("/")
    return addr if "://" in addr else "http://" + addr


class Balancer:
    """Backends of one role with their in-flight load.

    Backends can be added and removed while serving (the reference proxy's
    ``/instances/add`` and ``/instances/remove``); a backend removed while it
    still has requests in flight is isolated -- it gets no new ones -- and
    leaves once they are done.
    """

    def __init__(self, backends: list[str]):
        if not backends:
            raise ValueError("the proxy needs at least one backend")
        self.backends: list[str] = []
        self.inflight: dict[str, int] = {}
        self.load: dict[str, float] = {}
        self.served: dict[str, int] = {}
        self.isolated: set[str] = set()
        self._rr = 0
        self._lock = threading.Lock()
        for b in backends:
            self.add(b)

    def add(self, b: str) -> bool:
        b = normalize_url(b)
        with self._lock:
            self.isolated.discard(b)
            if b in self.inflight:
                return False
            self.backends.append(b)
            self.inflight[b], self.load[b], self.served[b] = 0, 0.0, 0
            return True

    def remove(self, b: str) -> str:
        """"removed", "isolated" (leaves when drained) or "unknown"."""
        b = normalize_url(b)
        with self._lock:
            if b not in self.inflight:
                return "unknown"
            if self.inflight[b] == 0:
                self._drop(b)
                return "removed"
            self.isolated.add(b)
            return "isolated"

    def _drop(self, b: str) -> None:
        self.backends.remove(b)
        self.isolated.discard(b)
        for d in (self.inflight, self.load, self.served):
            d.pop(b, None)

    def acquire(self, load: float = 1.0) -> str:
        with self._lock:
            live = [b for b in self.backends if b not in self.isolated]
            if not live:
                raise RuntimeError("no backend available")
            self._rr = (self._rr + 1) % len(live)
            order = live[self._rr:] + live[: self._rr]
            b = min(order, key=lambda x: (self.load[x], self.inflight[x]))
            self.inflight[b] += 1
            self.load[b] += load
            return b

    def release(self, b: str, load: float = 1.0) -> None:
        with self._lock:
            if b not in self.inflight:
                return
            self.inflight[b] -= 1
            self.load[b] = max(0.0, self.load[b] - load)
            self.served[b] += 1
            if b in self.isolated and self.inflight[b] == 0:
                self._drop(b)

    def snapshot(self) -> dict:
        with self._lock:
            return {"inflight": dict(self.inflight), "served": dict(self.served),
                    "isolated": sorted(self.isolated)}


def _prompt_len(body: dict) -> int:
    if "messages" in body:
        return max(1, sum(len(str(m.get("content", "")).encode("utf-8")) for m in body["messages"]))
    p = body.get("prompt", "")
    return max(1, len(p) if isinstance(p, list) else len(str(p).encode("utf-8")))


def build_prefill_request(body: dict) -> dict:
    """The prefill leg: one token, cache rows held for a decode server."""
    out = dict(body)
    out["kv_transfer_params"] = {"do_remote_decode": True, "do_remote_prefill": False}
    out["max_tokens"] = 1
    if "max_completion_tokens" in out:
        out["max_completion_tokens"] = 1
    out["stream"] = False
    return out


def _healthy(url: str, timeout_s: float = 2.0) -> bool:
    try:
        return requests.get(url + "/health", timeout=timeout_s).status_code == 200
    except requests.RequestException:
        return False


def build_proxy_app(backends: list[str] | None = None, *, prefill: list[str] | None = None,
                    decode: list[str] | None = None, timeout_s: float = 600.0, max_retries: int = 3,
                    retry_delay_s: float = 0.2, instance_retry_s: float = 5.0, instance_retry_max: int = 60):
    """``max_retries`` / ``retry_delay_s``: a backend that cannot be reached is
    retried with exponential back-off (``tools/proxy_server.py:869-892``).
    Instances added while unhealthy wait and are checked every
    ``instance_retry_s`` up to ``instance_retry_max`` times."""
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, StreamingResponse

    pd = bool(prefill or decode)
    if pd and not (prefill and decode):
        raise ValueError("disaggregated mode needs both prefill and decode servers")
    if pd and backends:
        raise ValueError("give either backends or prefill + decode servers")
    pools = {"prefill": Balancer(prefill), "decode": Balancer(decode)} if pd else {"backend": Balancer(backends or [])}
    app = FastAPI(title="afd_plugin_b200 proxy")
    app.state.pools = pools
    app.state.balancer = pools.get("backend")

    def _post(url: str, body: dict, *, stream: bool = False):
        import time

        for attempt in range(1, max_retries + 1):
            try:
                return requests.post(url, json=body, timeout=timeout_s, stream=stream)
            except requests.ConnectionError as exc:
                if attempt == max_retries:
                    raise HTTPException(status_code=502, detail=f"backend {url} failed: {exc}") from exc
                time.sleep(retry_delay_s * 2 ** (attempt - 1))
            except requests.RequestException as exc:
                raise HTTPException(status_code=502, detail=f"backend {url} failed: {exc}") from exc
        raise AssertionError("unreachable")

    waiting: dict[tuple[str, str], int] = {}  # (role, url) -> checks so far
    waiting_lock = threading.Lock()

    def _retry_waiting():
        import time

        while True:
            time.sleep(instance_retry_s)
            with waiting_lock:
                items = list(waiting.items())
            for (role, url), tries in items:
                ok = _healthy(url)
                with waiting_lock:
                    if ok:
                        pools[role].add(url)
                        waiting.pop((role, url), None)
                    elif tries + 1 >= instance_retry_max:
                        waiting.pop((role, url), None)
                    else:
                        waiting[(role, url)] = tries + 1

    threading.Thread(target=_retry_waiting, name="afd-proxy-instances", daemon=True).start()

    def _instances():
        out = {f"current_{role}_instances": list(bal.backends) for role, bal in pools.items()}
        with waiting_lock:
            out["waiting_instances"] = [f"{role}:{url}" for role, url in waiting]
        return out

    def _answer(r, release):
        """JSON answers are read whole; event streams are relayed chunk by chunk.

        ``release`` runs once the backend's answer has been consumed.
        """
        if r.status_code != 200 or not r.headers.get("content-type", "").startswith("text/event-stream"):
            try:
                return JSONResponse(status_code=r.status_code, content=r.json())
            finally:
                r.close()
                release()

        async def relay():
            # on the event loop, so a client disconnect cancels it at the next
            # await; closing the backend connection then aborts the request there
            import anyio

            chunks = r.iter_content(chunk_size=None)
            try:
                while True:
                    chunk = await anyio.to_thread.run_sync(next, chunks, None)
                    if chunk is None:
                        break
                    if chunk:
                        yield chunk
            finally:
                r.close()
                release()

        return StreamingResponse(relay(), media_type="text/event-stream")

    def _acquire(bal: Balancer, load: float = 1.0) -> str:
        try:
            return bal.acquire(load)
        except RuntimeError as exc:
            raise HTTPException(status_code=503, detail=str(exc)) from exc

    def _plain(body: dict, path: str):
        bal = pools["backend"]
        b = _acquire(bal)
        try:
            r = _post(b + path, body, stream=bool(body.get("stream")))
        except BaseException:
            bal.release(b)
            raise
        return _answer(r, lambda: bal.release(b))

    def _disaggregated(body: dict, path: str):
        pre, dec = pools["prefill"], pools["decode"]
        n_prompt = float(_prompt_len(body))
        p = _acquire(pre, n_prompt)
        try:
            r1 = _post(p + path, build_prefill_request(body))
        finally:
            pre.release(p, n_prompt)
        if r1.status_code != 200:
            return JSONResponse(status_code=r1.status_code, content=r1.json())
        params = r1.json().get("kv_transfer_params")
        if not params:
            raise HTTPException(status_code=502, detail=f"prefill server {p} returned no kv_transfer_params")
        n_dec = float(body.get("max_tokens", 16))
        d = _acquire(dec, n_dec)

        def drop_held_rows():  # the decode side never fetched the rows: free them now
            try:
                requests.delete(f"{p}/v1/kv/{params['remote_request_id']}", timeout=10)
            except requests.RequestException:
                pass

        try:
            r2 = _post(d + path, dict(body, kv_transfer_params=params), stream=bool(body.get("stream")))
        except BaseException:
            dec.release(d, n_dec)
            drop_held_rows()
            raise
        if r2.status_code != 200:
            drop_held_rows()
        return _answer(r2, lambda: dec.release(d, n_dec))

    @app.post("/instances/add")
    async def add_instances(request: Request):
        """``{"type": "prefill" | "decode" | "backend", "instances": ["host:port", ...]}``;
        unhealthy instances wait and are added once ``/health`` answers."""
        import anyio

        req = await request.json()
        role = req.get("type", "" if pd else "backend")
        if role not in pools:
            return JSONResponse(status_code=400, content={"error": f"instance type {role!r} is not one of {sorted(pools)}"})
        urls = [normalize_url(u) for u in ([req["instances"]] if isinstance(req.get("instances"), str)
                                           else req.get("instances", []))]
        added, queued = [], []
        for u in urls:
            if await anyio.to_thread.run_sync(_healthy, u):
                pools[role].add(u)
                added.append(u)
            else:
                with waiting_lock:
                    waiting[(role, u)] = 0
                queued.append(u)
        return dict(_instances(), added=added, waiting_to_be_added=queued)

    @app.post("/instances/remove")
    async def remove_instances(request: Request):
        """``{"type": ..., "instances": [...]}``; busy instances are isolated and leave when drained."""
        req = await request.json()
        role = req.get("type", "" if pd else "backend")
        if role not in pools:
            return JSONResponse(status_code=400, content={"error": f"instance type {role!r} is not one of {sorted(pools)}"})
        urls = [normalize_url(u) for u in ([req["instances"]] if isinstance(req.get("instances"), str)
                                           else req.get("instances", []))]
        result = {u: pools[role].remove(u) for u in urls}
        with waiting_lock:
            for u in urls:
                if waiting.pop((role, u), None) is not None:
                    result[u] = "removed"
        return dict(_instances(), result=result)

    @app.post("/reset_prefix_cache")
    def reset_prefix_cache():
        out = {}
        for bal in pools.values():
            for b in bal.backends:
                try:
                    out[b] = requests.post(b + "/reset_prefix_cache", timeout=10).json()
                except (requests.RequestException, ValueError) as exc:
                    out[b] = {"error": repr(exc)}
        return out

    @app.get("/healthcheck")
    def healthcheck():
        return health()

    @app.get("/v1/models")
    def models():
        """The model list of the first reachable backend (every backend serves the same model)."""
        for bal in pools.values():
            for b in bal.backends:
                try:
                    r = requests.get(b + "/v1/models", timeout=5)
                    if r.status_code == 200:
                        return r.json()
                except requests.RequestException:
                    continue
        raise HTTPException(status_code=503, detail="no backend answered /v1/models")

    @app.get("/health")
    def health():
        out = {}
        for name, bal in pools.items():
            status = {}
            for b in bal.backends:
                try:
                    status[b] = requests.get(b + "/health", timeout=2).ok
                except requests.RequestException:
                    status[b] = False
            out[name] = dict(bal.snapshot(), backends=status)
        if not pd:  # flat layout for the single-pool proxy
            out = out["backend"]
        return out

    async def _route(request: Request, path: str):
        import anyio

        body = await request.json()
        return await anyio.to_thread.run_sync(lambda: (_disaggregated if pd else _plain)(body, path))

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await _route(request, "/v1/completions")

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        return await _route(request, "/v1/chat/completions")

    return app


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="load-balancing / prefill-decode proxy over completion servers")
    ap.add_argument("--backends", default="", help="comma-separated base URLs (aggregated serving)")
    ap.add_argument("--prefill", default="", help="comma-separated prefill server URLs")
    ap.add_argument("--decode", default="", help="comma-separated decode server URLs")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-retries", type=int, default=3)
    ap.add_argument("--retry-delay", type=float, default=0.2)
    args = ap.parse_args(argv)
    import uvicorn

    split = lambda s: [x for x in s.split(",") if x]  # noqa: E731
    app = build_proxy_app(split(args.backends) or None, prefill=split(args.prefill) or None,
                          decode=split(args.decode) or None, max_retries=args.max_retries,
                          retry_delay_s=args.retry_delay)
    uvicorn.run(app, host=args.host, port=args.port)


if __name__ == "__main__":
    main()
