"""Online serving benchmark against a completions server or the proxy.

    python -m afd_plugin_b200.bench.serve_bench --url http://127.0.0.1:8000 \\
        --num-prompts 1024 --input-len 1024 --output-len 128 --request-rate 5 --max-concurrency 32

The load the reference's launch scripts drive through ``vllm bench serve``
(``tools/benchmarks/request_generator.sh:15-57``: ISL 1024, OSL 128, 1024
prompts, rate 5, concurrency 32).  Requests carry random token ids, arrive as
a Poisson process at ``--request-rate`` per second (``inf``: all at once) with
at most ``--max-concurrency`` in flight, and stream their tokens
(``"stream": true``), so time to first token (TTFT), time per output token
after the first (TPOT), inter-token latency (ITL) and end-to-end latency are
measured per request on the client.  Prints one JSON summary.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from dataclasses import dataclass, field


@dataclass
class RequestResult:
    ok: bool = False
    prompt_len: int = 0
    output_tokens: int = 0
    ttft_s: float = 0.0
    latency_s: float = 0.0
    itl_s: list[float] = field(default_factory=list)
    error: str = ""


def _pct(values: list[float], q: float) -> float:
    if not values:
        return 0.0
    v = sorted(values)
    return v[min(len(v) - 1, int(q * (len(v) - 1) + 0.5))]


def _stats(name: str, values_s: list[float]) -> dict:
    ms = [x * 1e3 for x in values_s]
    return {f"mean_{name}_ms": round(sum(ms) / len(ms), 3) if ms else 0.0,
            f"median_{name}_ms": round(_pct(ms, 0.5), 3), f"p99_{name}_ms": round(_pct(ms, 0.99), 3)}


async def _one(session, url: str, prompt: list[int], max_tokens: int, timeout_s: float) -> RequestResult:
    import aiohttp

    res = RequestResult(prompt_len=len(prompt))
    t0 = time.perf_counter()
    last = t0
    try:
        async with session.post(url, json={"prompt": prompt, "max_tokens": max_tokens, "stream": True},
                                timeout=aiohttp.ClientTimeout(total=timeout_s)) as r:
            if r.status != 200:
                res.error = f"HTTP {r.status}: {(await r.text())[:200]}"
                return res
            buf = b""
            async for chunk in r.content.iter_any():
                buf += chunk
                while b"\n\n" in buf:
                    event, buf = buf.split(b"\n\n", 1)
                    line = event.decode().strip()
                    if not line.startswith("data: "):
                        continue
                    data = line[len("data: "):]
                    if data == "[DONE]":
                        continue
                    msg = json.loads(data)
                    if "error" in msg:
                        res.error = msg["error"].get("message", "stream error")
                        return res
                    n = sum(len(c.get("token_ids", [])) for c in msg.get("choices", []))
                    if n:
                        now = time.perf_counter()
                        if res.output_tokens == 0:
                            res.ttft_s = now - t0
                        else:
                            res.itl_s.append(now - last)
                        last = now
                        res.output_tokens += n
        res.latency_s = time.perf_counter() - t0
        res.ok = res.output_tokens > 0
    except Exception as exc:  # noqa: BLE001 - counted as a failed request
        res.error = repr(exc)
    return res


async def run(url: str, prompts: list[list[int]], max_tokens: int, *, request_rate: float, max_concurrency: int,
              seed: int = 0, timeout_s: float = 600.0) -> dict:
    import aiohttp

    endpoint = url.rstrip("/") + "/v1/completions"
    rng = random.Random(seed)
    sem = asyncio.Semaphore(max(1, max_concurrency))

    async def limited(session, p):
        async with sem:
            return await _one(session, endpoint, p, max_tokens, timeout_s)

    t0 = time.perf_counter()
    async with aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=0)) as session:
        tasks = []
        for p in prompts:
            tasks.append(asyncio.create_task(limited(session, p)))
            if request_rate != float("inf"):
                await asyncio.sleep(rng.expovariate(request_rate))
        results = await asyncio.gather(*tasks)
    duration = time.perf_counter() - t0
    done = [r for r in results if r.ok]
    out_tokens = sum(r.output_tokens for r in done)
    in_tokens = sum(r.prompt_len for r in done)
    tpot = [(r.latency_s - r.ttft_s) / (r.output_tokens - 1) for r in done if r.output_tokens > 1]
    summary = {
        "completed": len(done), "failed": len(results) - len(done), "duration_s": round(duration, 3),
        "request_throughput": round(len(done) / duration, 3),
        "output_throughput_tok_s": round(out_tokens / duration, 2),
        "total_token_throughput_tok_s": round((in_tokens + out_tokens) / duration, 2),
        "total_input_tokens": in_tokens, "total_output_tokens": out_tokens,
        **_stats("ttft", [r.ttft_s for r in done]), **_stats("tpot", tpot),
        **_stats("itl", [x for r in done for x in r.itl_s]), **_stats("e2el", [r.latency_s for r in done]),
        "request_rate": request_rate, "max_concurrency": max_concurrency,
    }
    errors = [r.error for r in results if not r.ok]
    if errors:
        summary["first_error"] = errors[0]
    return summary


def make_prompts(n: int, input_len: int, vocab: int, seed: int = 0) -> list[list[int]]:
    rng = random.Random(seed)
    return [[rng.randrange(vocab) for _ in range(input_len)] for _ in range(n)]


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--num-prompts", type=int, default=1024)
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=128)
    ap.add_argument("--request-rate", type=float, default=5.0, help="requests/s (inf: all at once)")
    ap.add_argument("--max-concurrency", type=int, default=32)
    ap.add_argument("--vocab-size", type=int, default=32000, help="token ids are drawn below this")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--timeout", type=float, default=600.0)
    ap.add_argument("--output", default=None, help="also write the summary JSON here")
    args = ap.parse_args(argv)
    prompts = make_prompts(args.num_prompts, args.input_len, args.vocab_size, args.seed)
    summary = asyncio.run(run(args.url, prompts, args.output_len, request_rate=args.request_rate,
                              max_concurrency=args.max_concurrency, seed=args.seed, timeout_s=args.timeout))
    summary.update(num_prompts=args.num_prompts, input_len=args.input_len, output_len=args.output_len)
    print(json.dumps(summary), flush=True)
    if args.output:
        with open(args.output, "w") as fh:
            json.dump(summary, fh)
    return summary


if __name__ == "__main__":
    main()
