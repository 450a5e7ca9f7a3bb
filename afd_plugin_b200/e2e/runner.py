"""End-to-end scenario runner: serve, send requests, compare against a baseline, tear down.

    python -m afd_plugin_b200.e2e.runner --scenarios baseline-graph,afd-graph-2a2f,afd-fused-graph-2a2f \\
        --preset deepseek-v2-lite --devices 0,1,2,3 --output e2e.json

Each scenario's server (``python -m afd_plugin_b200.serving``, under
``torch.distributed.run`` for AFD worlds) runs in its own process group
(``process_utils``).  The runner waits for ``/health``, sends a fixed set of
token-id prompts (seeded, so every scenario sees the same requests) with
bounded concurrency, records the greedy outputs, and stops the group.

Gate: the first scenario is the reference; every later one must reproduce its
first tokens for at least ``--min-first-token-match`` of the requests and its
whole outputs for at least ``--min-exact-match`` -- a disaggregated deployment
must match the colocated engine token for token when it computes the same
math (fp32, or bf16 up to reduction order).  With ``--gsm8k-data`` every
scenario is also gated on GSM8K accuracy (``e2e/gsm8k.py``), the reference's
gate (``docs/design/module/e2e_testing.md:145-163``); that needs a real
checkpoint and a local copy of the dataset.
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import sys
import time
from concurrent.futures import ThreadPoolExecutor

import requests

from afd_plugin_b200.e2e.process_utils import start_server, stop_server, wait_for_health
from afd_plugin_b200.e2e.scenarios import SCENARIOS, Scenario, server_command


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_prompts(n: int, vocab: int, *, seed: int = 0, min_len: int = 8, max_len: int = 64) -> list[list[int]]:
    import random

    rng = random.Random(seed)
    return [[rng.randrange(vocab) for _ in range(rng.randint(min_len, max_len))] for _ in range(n)]


def send_requests(url: str, prompts: list[list[int]], max_tokens: int, *, concurrency: int = 8,
                  timeout_s: float = 600.0) -> list[list[int]]:
    def one(p):
        r = requests.post(url.rstrip("/") + "/v1/completions", json={"prompt": p, "max_tokens": max_tokens},
                          timeout=timeout_s)
        r.raise_for_status()
        return r.json()["choices"][0]["token_ids"]

    with ThreadPoolExecutor(max(1, concurrency)) as ex:
        return list(ex.map(one, prompts))


def compare(outputs: list[list[int]], reference: list[list[int]]) -> dict:
    """Agreement of ``outputs`` with ``reference`` (same prompts, same order)."""
    if len(outputs) != len(reference):
        raise ValueError("output and reference request counts differ")
    n = max(1, len(reference))
    exact = sum(o == r for o, r in zip(outputs, reference))
    first = sum(bool(o) and bool(r) and o[0] == r[0] for o, r in zip(outputs, reference))
    prefix = 0.0
    for o, r in zip(outputs, reference):
        k = 0
        while k < min(len(o), len(r)) and o[k] == r[k]:
            k += 1
        prefix += k / max(1, len(r))
    return {"exact_match": exact / n, "first_token_match": first / n, "mean_prefix_agreement": prefix / n}


def gate(metrics: dict, *, min_exact: float, min_first: float) -> list[str]:
    """Reasons the comparison fails the gate (empty: passed)."""
    bad = []
    if metrics["exact_match"] < min_exact:
        bad.append(f"exact_match {metrics['exact_match']:.3f} < {min_exact}")
    if metrics["first_token_match"] < min_first:
        bad.append(f"first_token_match {metrics['first_token_match']:.3f} < {min_first}")
    return bad


_PORT_TAKEN = ("address already in use", "EADDRINUSE", "error while attempting to bind")


def run_scenario(scn: Scenario, args, prompts: list[list[int]], *, log_dir: str, attempts: int = 3) -> dict:
    """Serve ``scn`` and run the prompts; a server that lost its probed port to
    another process is started again on fresh ports (up to ``attempts`` times)."""
    for attempt in range(1, attempts + 1):
        try:
            return _run_scenario_once(scn, args, prompts, log_dir=log_dir)
        except RuntimeError as exc:
            if attempt == attempts or not any(m in str(exc) for m in _PORT_TAKEN):
                raise
    raise AssertionError("unreachable")


def _server_env(args, devices: list[str] | None) -> dict:
    env = dict(os.environ)
    # the servers import this package from the same tree as the runner
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    env["PYTHONPATH"] = os.pathsep.join([root] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    if args.device == "cpu":
        env["CUDA_VISIBLE_DEVICES"] = ""
    elif devices is not None:
        env["CUDA_VISIBLE_DEVICES"] = ",".join(devices)
    return env


def _launch(scn: Scenario, args, log_path: str, devices: list[str] | None):
    port, master = free_port(), free_port()
    cmd = server_command(scn, python=sys.executable, preset=args.preset, port=port, master_port=master,
                         checkpoint=args.checkpoint, dtype=args.dtype, max_num_seqs=args.max_num_seqs,
                         max_model_len=args.max_model_len, capture_size=args.capture_size, seed=args.seed)
    server = start_server(cmd, env=_server_env(args, devices), log_path=log_path)
    return server, f"http://127.0.0.1:{port}", cmd


def _run_scenario_once(scn: Scenario, args, prompts: list[list[int]], *, log_dir: str) -> dict:
    from dataclasses import replace

    all_devices = [d for d in args.devices.split(",") if d] if args.devices else None
    if all_devices is None and args.device == "cuda" and scn.prefill is not None:
        all_devices = [str(i) for i in range(scn.total_devices)]
    servers = []
    result = {"scenario": scn.name}
    try:
        if scn.prefill is None:
            server, url, cmd = _launch(scn, args, os.path.join(log_dir, f"{scn.name}.log"), all_devices)
            servers.append(server)
            result.update(cmd=cmd, log=server.log_path)
        else:
            # disjoint devices: the prefill server first, then the decode deployment
            n_pre = scn.prefill.world_size
            pre_dev = all_devices[:n_pre] if all_devices else None
            dec_dev = all_devices[n_pre:] if all_devices else None
            pre, pre_url, _ = _launch(scn.prefill, args, os.path.join(log_dir, f"{scn.name}.prefill.log"), pre_dev)
            servers.append(pre)
            dec, dec_url, cmd = _launch(replace(scn, prefill=None), args,
                                        os.path.join(log_dir, f"{scn.name}.decode.log"), dec_dev)
            servers.append(dec)
            wait_for_health(pre, pre_url, timeout_s=args.startup_timeout)
            wait_for_health(dec, dec_url, timeout_s=args.startup_timeout)
            pport = free_port()
            proxy = start_server([sys.executable, "-m", "afd_plugin_b200.serving.proxy", "--prefill", pre_url,
                                  "--decode", dec_url, "--port", str(pport)], env=_server_env(args, []),
                                 log_path=os.path.join(log_dir, f"{scn.name}.proxy.log"))
            servers.append(proxy)
            server, url = proxy, f"http://127.0.0.1:{pport}"
            result.update(cmd=cmd, log=dec.log_path)
        result["startup_s"] = round(wait_for_health(server, url, timeout_s=args.startup_timeout), 2)
        t0 = time.perf_counter()
        outs = send_requests(url, prompts, args.max_tokens, concurrency=args.concurrency,
                             timeout_s=args.request_timeout)
        dt = time.perf_counter() - t0
        result.update(outputs=outs, wall_s=round(dt, 3),
                      output_tok_per_s=round(sum(len(o) for o in outs) / max(dt, 1e-9), 1))
        if args.gsm8k_data:
            from afd_plugin_b200.e2e import gsm8k

            data = gsm8k.load_jsonl(args.gsm8k_data)
            pool = gsm8k.load_jsonl(args.gsm8k_train) if args.gsm8k_train else data
            shots = pool[: args.gsm8k_shots]
            if not args.gsm8k_train:
                data = data[args.gsm8k_shots:]
            result["gsm8k"] = gsm8k.evaluate(url, data, shots, limit=args.gsm8k_limit,
                                             timeout_s=args.request_timeout)
    finally:
        result["teardown"] = ",".join(stop_server(s_) for s_ in reversed(servers))
    return result


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--scenarios", default="baseline-graph,afd-graph-2a2f",
                    help=f"comma-separated, first one is the reference; known: {', '.join(SCENARIOS)}")
    ap.add_argument("--preset", default="deepseek-v2-lite")
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"])
    ap.add_argument("--devices", default="", help="CUDA_VISIBLE_DEVICES for the servers")
    ap.add_argument("--num-prompts", type=int, default=16)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--min-prompt-len", type=int, default=8)
    ap.add_argument("--max-prompt-len", type=int, default=64)
    ap.add_argument("--concurrency", type=int, default=8)
    ap.add_argument("--max-num-seqs", type=int, default=16)
    ap.add_argument("--max-model-len", type=int, default=2048)
    ap.add_argument("--capture-size", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--startup-timeout", type=float, default=900.0)
    ap.add_argument("--request-timeout", type=float, default=600.0)
    ap.add_argument("--min-exact-match", type=float, default=0.0)
    ap.add_argument("--min-first-token-match", type=float, default=0.9)
    ap.add_argument("--gsm8k-data", default=None, help="GSM8K test JSONL: also gate every scenario on accuracy")
    ap.add_argument("--gsm8k-train", default=None, help="few-shot examples JSONL (default: head of --gsm8k-data)")
    ap.add_argument("--gsm8k-shots", type=int, default=8)
    ap.add_argument("--gsm8k-limit", type=int, default=7)
    ap.add_argument("--gsm8k-threshold", type=float, default=0.27)
    ap.add_argument("--log-dir", default="e2e_logs")
    ap.add_argument("--output", default=None, help="write the results as JSON here")
    args = ap.parse_args(argv)

    names = [s for s in args.scenarios.split(",") if s]
    unknown = [s for s in names if s not in SCENARIOS]
    if unknown:
        ap.error(f"unknown scenarios {unknown}")
    scns = [SCENARIOS[s] for s in names]
    if args.device == "cpu" and any(s.needs_cuda for s in scns):
        ap.error("the fused connector scenarios need CUDA devices")
    from afd_plugin_b200.models.configs import get_preset

    vocab = get_preset(args.preset).vocab_size
    prompts = make_prompts(args.num_prompts, vocab, seed=args.seed, min_len=args.min_prompt_len,
                           max_len=args.max_prompt_len)
    os.makedirs(args.log_dir, exist_ok=True)
    results, failures = [], []
    for scn in scns:
        try:
            res = run_scenario(scn, args, prompts, log_dir=args.log_dir)
        except Exception as exc:  # noqa: BLE001 - recorded, the other scenarios still run
            res = {"scenario": scn.name, "error": repr(exc)}
            failures.append(f"{scn.name}: {exc!r}")
        results.append(res)
        print(json.dumps({k: v for k, v in res.items() if k not in ("outputs", "cmd")}), flush=True)
    for res in results:
        g = res.get("gsm8k")
        if g is not None and g["exact_match_flexible"] < args.gsm8k_threshold:
            failures.append(f"{res['scenario']}: gsm8k {g['exact_match_flexible']:.3f} < {args.gsm8k_threshold}")
    ref = results[0].get("outputs")
    for res in results[1:]:
        if ref is None or "outputs" not in res:
            continue
        res["agreement"] = compare(res["outputs"], ref)
        bad = gate(res["agreement"], min_exact=args.min_exact_match, min_first=args.min_first_token_match)
        res["gate"] = "pass" if not bad else "fail: " + "; ".join(bad)
        failures += [f"{res['scenario']}: {b}" for b in bad]
        print(json.dumps({"scenario": res["scenario"], "agreement": res["agreement"], "gate": res["gate"]}),
              flush=True)
    if args.output:
        with open(args.output, "w") as fh:
            json.dump({"preset": args.preset, "dtype": args.dtype, "prompts": prompts, "results": results}, fh)
    for f in failures:
        print("FAIL", f, file=sys.stderr)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
