"""Load-balancing proxy in front of several completion servers.

Routes each ``POST /v1/completions`` to the backend with the fewest requests
in flight (ties: round robin) and forwards the JSON answer; ``GET /health``
reports the backends.  The counterpart of the reference's proxy tool
(``tools/proxy_server.py``) for data-parallel serving instances; the
prefill -> decode KV hand-off that tool also drives (through LMCache) is not
part of this framework.

    python -m afd_plugin_b200.serving.proxy --backends http://127.0.0.1:8001,http://127.0.0.1:8002 --port 8000
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
        self.served = {b: 0 for b in self.backends}
        self._rr = itertools.cycle(range(len(self.backends)))
        self._lock = threading.Lock()

    def acquire(self) -> str:
        with self._lock:
            start = next(self._rr)
            order = self.backends[start:] + self.backends[:start]
            b = min(order, key=lambda x: self.inflight[x])
            self.inflight[b] += 1
            return b

    def release(self, b: str) -> None:
        with self._lock:
            self.inflight[b] -= 1
            self.served[b] += 1


def build_proxy_app(backends: list[str], *, timeout_s: float = 600.0):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse

    bal = Balancer(backends)
    app = FastAPI(title="afd_plugin_b200 proxy")
    app.state.balancer = bal

    @app.get("/health")
    def health():
        status = {}
        for b in bal.backends:
            try:
                status[b] = requests.get(b + "/health", timeout=2).ok
            except requests.RequestException:
                status[b] = False
        return {"backends": status, "inflight": dict(bal.inflight), "served": dict(bal.served)}

    @app.post("/v1/completions")
    async def completions(request: Request):
        body = await request.json()
        b = bal.acquire()
        try:
            import anyio

            r = await anyio.to_thread.run_sync(lambda: requests.post(b + "/v1/completions", json=body,
                                                                     timeout=timeout_s))
        except requests.RequestException as exc:
            raise HTTPException(status_code=502, detail=f"backend {b} failed: {exc}") from exc
        finally:
            bal.release(b)
        return JSONResponse(status_code=r.status_code, content=r.json())

    return app


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="least-loaded proxy over completion servers")
    ap.add_argument("--backends", required=True, help="comma-separated base URLs")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    args = ap.parse_args(argv)
    import uvicorn

    uvicorn.run(build_proxy_app(args.backends.split(",")), host=args.host, port=args.port)


if __name__ == "__main__":
    main()
