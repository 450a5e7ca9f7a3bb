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
disaggregated mode only the decode leg streams.  ``GET /health`` reports
every backend.

    python -m afd_plugin_b200.serving.proxy --backends http://127.0.0.1:8001,http://127.0.0.1:8002 --port 8000
    python -m afd_plugin_b200.serving.proxy --prefill http://127.0.0.1:8001 --decode http://127.0.0.1:8002
"""

from __future__ import annotations

import argparse
import itertools
import threading

import requests
from fastapi import Request


class Balancer:
    def __init__(self, backends: list[str]):
        if not backends:
            raise ValueError("the proxy needs at least one backend")
        self.backends = [b.rstrip("/") for b in backends]
        self.inflight = {b: 0 for b in self.backends}
        self.load = {b: 0.0 for b in self.backends}
        self.served = {b: 0 for b in self.backends}
        self._rr = itertools.cycle(range(len(self.backends)))
        self._lock = threading.Lock()

    def acquire(self, load: float = 1.0) -> str:
        with self._lock:
            start = next(self._rr)
            order = self.backends[start:] + self.backends[:start]
            b = min(order, key=lambda x: (self.load[x], self.inflight[x]))
            self.inflight[b] += 1
            self.load[b] += load
            return b

    def release(self, b: str, load: float = 1.0) -> None:
        with self._lock:
            self.inflight[b] -= 1
            self.load[b] = max(0.0, self.load[b] - load)
            self.served[b] += 1

    def snapshot(self) -> dict:
        with self._lock:
            return {"inflight": dict(self.inflight), "served": dict(self.served)}


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


def build_proxy_app(backends: list[str] | None = None, *, prefill: list[str] | None = None,
                    decode: list[str] | None = None, timeout_s: float = 600.0):
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
        try:
            return requests.post(url, json=body, timeout=timeout_s, stream=stream)
        except requests.RequestException as exc:
            raise HTTPException(status_code=502, detail=f"backend {url} failed: {exc}") from exc

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

    def _plain(body: dict, path: str):
        bal = pools["backend"]
        b = bal.acquire()
        try:
            r = _post(b + path, body, stream=bool(body.get("stream")))
        except BaseException:
            bal.release(b)
            raise
        return _answer(r, lambda: bal.release(b))

    def _disaggregated(body: dict, path: str):
        pre, dec = pools["prefill"], pools["decode"]
        n_prompt = float(_prompt_len(body))
        p = pre.acquire(n_prompt)
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
        d = dec.acquire(n_dec)

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
    args = ap.parse_args(argv)
    import uvicorn

    split = lambda s: [x for x in s.split(",") if x]  # noqa: E731
    app = build_proxy_app(split(args.backends) or None, prefill=split(args.prefill) or None,
                          decode=split(args.decode) or None)
    uvicorn.run(app, host=args.host, port=args.port)


if __name__ == "__main__":
    main()
