"""Serve completions over HTTP.

Colocated (one process):
    python -m afd_plugin_b200.serving --preset tiny-dsv2 --port 8000

AFD (one process per GPU; Attention rank 0 serves HTTP; ``--tp`` shards the
attention heads over consecutive Attention ranks), either as one torchrun
world of A + F ranks:
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m afd_plugin_b200.serving \\
        --preset deepseek-v2-lite --afd '{"num_attention_ranks": 1, "num_ffn_ranks": 1,
                                          "connector": "B200FusedAFDConnector"}'

or one launch per role, the way the reference deploys two ``vllm serve``
instances: each launch gives its ``role`` and the AFD world's ``host`` /
``port``, and its ranks join that world (FFN ranks first)::

    torchrun --nproc-per-node 2 -m afd_plugin_b200.serving --afd \\
        '{"role": "ffn", "num_attention_ranks": 6, "num_ffn_ranks": 2, "host": "10.0.0.1", "port": 1239}'
    torchrun --nproc-per-node 6 -m afd_plugin_b200.serving --port 8000 --afd \\
        '{"role": "attention", "num_attention_ranks": 6, "num_ffn_ranks": 2, "host": "10.0.0.1", "port": 1239}'
"""

from __future__ import annotations

import argparse
import json
import os


def parse_args(argv=None) -> argparse.Namespace:
    """Server flags; the vLLM spellings used by the reference's launch recipes are accepted too.

    ``--additional-config '{"afd": {...}}'`` (the reference's AFD switch),
    ``--compilation-config '{"cudagraph_mode": "FULL_DECODE_ONLY", "cudagraph_capture_sizes": [...]}'``,
    ``--enforce-eager``, ``--enable-dbo``, ``--tensor-parallel-size``,
    ``--model`` / a positional model path, ``--served-model-name``;
    ``--enable-expert-parallel`` and the DBO token thresholds are accepted and
    have nothing to switch (FFN ranks always shard experts; DBO splits any
    batch of two or more).
    """
    ap = argparse.ArgumentParser(description="afd_plugin_b200 completions server")
    ap.add_argument("model_path", nargs="?", default=None, help="HF checkpoint directory (as `vllm serve MODEL`)")
    ap.add_argument("--preset", default="tiny-dsv2", help="architecture when no checkpoint is given")
    ap.add_argument("--checkpoint", "--model", dest="checkpoint", default=None,
                    help="HF safetensors directory (random init when absent)")
    ap.add_argument("--tokenizer", default=None,
                    help="HF tokenizer directory (default: the checkpoint's; byte tokens when there is none)")
    ap.add_argument("--served-model-name", default="afd-b200")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--afd", default="", help='JSON additional_config["afd"] (empty: colocated)')
    ap.add_argument("--additional-config", default="", help='JSON {"afd": {...}} (the reference\'s switch)')
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--max-num-batched-tokens", type=int, default=None,
                    help="prompt tokens per prefill step (chunked prefill; default: whole prompts)")
    ap.add_argument("--eager", "--enforce-eager", dest="eager", action="store_true")
    ap.add_argument("--async-scheduling", action="store_true",
                    help="launch each greedy decode step before the previous step's tokens are read back")
    ap.add_argument("--capture-sizes", default="", help="comma-separated decode graph batch sizes "
                    "(default: --max-num-seqs)")
    ap.add_argument("--compilation-config", default="", help="JSON with cudagraph_mode / cudagraph_capture_sizes")
    ap.add_argument("--dbo", "--enable-dbo", dest="dbo", action="store_true",
                    help="two-ubatch overlap of attention and FFN (AFD only)")
    ap.add_argument("--dbo-decode-token-threshold", type=int, default=None)
    ap.add_argument("--dbo-prefill-token-threshold", type=int, default=None)
    ap.add_argument("--enable-expert-parallel", action="store_true")
    ap.add_argument("--enable-prefix-caching", action="store_true",
                    help="reuse the KV blocks of shared prompt prefixes (full-attention models)")
    ap.add_argument("--seed", type=int, default=0, help="random-init seed when no checkpoint is given")
    ap.add_argument("--decode-bench", action="store_true",
                    help="take every prompt as prefilled (random cache rows) and only decode: long-ISL decode "
                         "benchmarks without prefill")
    ap.add_argument("--tp", "--tensor-parallel-size", dest="tp", type=int, default=1,
                    help="attention tensor parallelism (AFD only; num_attention_ranks = DP x TP)")
    args = ap.parse_args(argv)
    if args.model_path and not args.checkpoint:
        args.checkpoint = args.model_path
    if args.additional_config:
        extra = json.loads(args.additional_config)
        if not isinstance(extra, dict):
            ap.error("--additional-config must be a JSON object")
        if "afd" in extra:
            if args.afd:
                ap.error("give the AFD config once: --afd or --additional-config")
            args.afd = json.dumps(extra["afd"])
    sizes = [int(x) for x in args.capture_sizes.split(",") if x]
    if args.compilation_config:
        cc = json.loads(args.compilation_config)
        mode = cc.get("cudagraph_mode")
        if mode not in (None, "FULL_DECODE_ONLY", "NONE"):
            ap.error(f"cudagraph_mode {mode!r}: only FULL_DECODE_ONLY (or NONE) is supported")
        if mode == "NONE":
            args.eager = True
        sizes = sizes or [int(x) for x in cc.get("cudagraph_capture_sizes", [])]
    args.sizes = sizes or [args.max_num_seqs]
    return args


def main(argv=None) -> None:
    args = parse_args(argv)
    sizes = args.sizes

    import torch
    import uvicorn

    from afd_plugin_b200.engine_config import CacheConfig, CompilationConfig, EngineConfig, ModelConfig, ParallelConfig
    from afd_plugin_b200.models.configs import get_preset
    from afd_plugin_b200.serving.api_server import EngineLoop, build_app
    from afd_plugin_b200.serving.tokenizer import load_tokenizer

    if args.checkpoint:
        from afd_plugin_b200.models.loader import read_hf_config

        arch = read_hf_config(args.checkpoint)
    else:
        arch = get_preset(args.preset)
    dtype = getattr(torch, args.dtype)
    afd = json.loads(args.afd) if args.afd else {}
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not afd:
        from afd_plugin_b200.runtime.engine import LLMEngine

        ec = EngineConfig(ModelConfig(arch, dtype=dtype, enforce_eager=args.eager, max_model_len=args.max_model_len,
                                      checkpoint=args.checkpoint, seed=args.seed),
                          compilation_config=CompilationConfig(cudagraph_capture_sizes=sizes),
                          cache_config=CacheConfig(enable_prefix_caching=args.enable_prefix_caching),
                          max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
                          async_scheduling=args.async_scheduling)
        engine = LLMEngine.colocated(ec, device="cuda" if torch.cuda.is_available() else "cpu")
        if not args.eager and engine.device.type == "cuda":
            engine.capture_graphs()
        if args.decode_bench:
            engine.kv.fill_random_(seed=args.seed)
        loop = EngineLoop(engine, decode_bench=args.decode_bench).start()
        uvicorn.run(build_app(loop, advertise_host=args.host, advertise_port=args.port,
                              model_name=args.served_model_name,
                              tokenizer=load_tokenizer(args.tokenizer or args.checkpoint, arch.vocab_size)),
                    host=args.host, port=args.port)
        return

    import torch.distributed as dist

    from afd_plugin_b200.parallel.topology import role_of_world_rank
    from afd_plugin_b200.runtime.workers import AFDAttentionWorker, AFDFFNWorker

    from afd_plugin_b200.config import afd_config_from_mapping
    from afd_plugin_b200.parallel.process_group import init_afd_world

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    A, F = int(afd["num_attention_ranks"]), int(afd["num_ffn_ranks"])
    given_role = afd.get("role", afd.get("afd_role"))
    per_role = given_role in ("attention", "ffn") and world == (A if given_role == "attention" else F)
    if per_role:
        # One role per launch, as the reference deploys (an Attention server and an FFN
        # server): this launch's ranks join the AFD world over tcp://host:port, FFN ranks first.
        cfg = afd_config_from_mapping(afd)
        rank = rank + (F if given_role == "attention" else 0)
        init_afd_world(backend=backend, host=cfg.host, port=cfg.port, world_size=A + F, rank=rank)
        world = A + F
    else:
        dist.init_process_group(backend=backend)
    if world != A + F:
        raise SystemExit(f"world size {world} != num_attention_ranks + num_ffn_ranks = {A + F}")
    if args.tp < 1 or A % args.tp:
        raise SystemExit(f"--tp {args.tp} must divide num_attention_ranks {A}")
    role, role_rank = role_of_world_rank(rank, attention_size=A, ffn_size=F)
    ec = EngineConfig(ModelConfig(arch, dtype=dtype, enforce_eager=args.eager, max_model_len=args.max_model_len,
                                  checkpoint=args.checkpoint, seed=args.seed),
                      parallel_config=ParallelConfig(data_parallel_size=A // args.tp, tensor_parallel_size=args.tp,
                                                     use_ubatching=args.dbo, num_ubatches=2 if args.dbo else 1),
                      compilation_config=CompilationConfig(cudagraph_capture_sizes=sizes),
                      cache_config=CacheConfig(enable_prefix_caching=args.enable_prefix_caching),
                      additional_config={"afd": dict(afd, role=role)}, max_num_seqs=args.max_num_seqs,
                      max_num_batched_tokens=args.max_num_batched_tokens, async_scheduling=args.async_scheduling)
    if role == "ffn":
        w = AFDFFNWorker(ec, local_rank=local)
        if per_role and role_rank == 0:
            # an FFN server launched on its own answers /health while its loop serves
            _serve_ffn_health(w, args.host, args.port)
        else:
            w.run_ffn_server_loop()
        w.shutdown()
        return
    w = AFDAttentionWorker(ec, local_rank=local)
    if not args.eager and backend == "nccl":
        w.engine.capture_graphs()
    if args.decode_bench:
        w.engine.kv.fill_random_(seed=args.seed)
    loop = EngineLoop(w.engine, group=w.groups.attention_group, world=A, rank=role_rank,
                      tp_group=w.groups.tp_cpu_group, tp_size=args.tp, tp_src=w.groups.tp_leader,
                      decode_bench=args.decode_bench).start()
    if role_rank == 0:
        uvicorn.run(build_app(loop, advertise_host=args.host, advertise_port=args.port,
                              model_name=args.served_model_name,
                              tokenizer=load_tokenizer(args.tokenizer or args.checkpoint, arch.vocab_size)),
                    host=args.host, port=args.port)
        loop.stop()  # every Attention rank's loop leaves at the same iteration
    else:
        loop.join()
    w.shutdown()  # stops the FFN ranks' serve loops


def _serve_ffn_health(worker, host: str, port: int) -> None:
    """Run the FFN loop on its thread and ``GET /health`` (200 while it serves) until it ends."""
    import threading
    import time

    import uvicorn
    from fastapi import FastAPI, HTTPException

    app = FastAPI(title="afd_plugin_b200 FFN")

    @app.get("/health")
    def health():
        if not worker.is_loop_alive():
            raise HTTPException(status_code=503, detail="FFN loop not running")
        return {"status": "ok", "role": "ffn"}

    worker.start_ffn_server_loop()
    server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level="warning"))

    def watch() -> None:  # the loop ends on the Attention side's shutdown: take the HTTP server down too
        while worker.is_loop_alive():
            time.sleep(0.2)
        server.should_exit = True

    threading.Thread(target=watch, name="afd-ffn-health-watch", daemon=True).start()
    server.run()
    worker.stop_ffn_server_loop()


if __name__ == "__main__":
    main()
