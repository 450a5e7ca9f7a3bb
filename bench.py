"""Decode-throughput benchmark (the driver contract).

    python bench.py --gpus N --steps K --warmup W [--impl reference]

Workload (the reference's DeepSeek-V2-Lite decode recipes): DeepSeek-V2-Lite architecture, bf16, random
init; 256 concurrent requests, 1024-token prompts, 256 output tokens.
Prompt KV is synthetic (filled at random, as the reference's decode-bench KV
connector does), so only decode steps run.  N=1 is colocated; N>1 runs AFD
with the FFN-first topology 1A1F (N=2), 2A2F (N=4), 4A4F (N=8)
(``--topology A,F`` overrides, e.g. 6,2).  The 256 requests are split over
the Attention ranks (fixed total work: strong scaling).

value   output tokens/s of the whole job, CUDA-event timed over exactly K
        decode steps (device-resident loop: graph replay + on-device input
        advance), max over ranks.
e2e     the same metric through the public engine API (``LLMEngine.step``):
        per step the host schedules, copies inputs host->device from pinned
        memory, replays, and reads the sampled tokens back.
Weights (~31 GB) and KV (~10 GB) are far larger than the 126 MB L2, so no L2
flush is needed between steps.

Diagnostics (not bench values): ``--phases`` adds per-role phase timing on the
device; ``AFD_BENCH_NVTX=1`` wraps the timed loop in an NVTX range named
"timed" (for a profiler's range filter); ``AFD_BENCH_VERBOSE=1`` logs each
rank's progress to stderr.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode output tok/s (8xB200, max over ranks) + p50 TPOT, AFD vs NCCL connector"
BASELINE_VALUE = None  # the reference publishes no GPU number for this metric
# (Attention ranks, FFN ranks) per GPU count.  With the batch fixed, a decode
# step is a per-layer chain of the Attention ranks' attention and the FFN
# ranks' expert GEMMs, and the FFN side is bound by streaming its experts'
# weights: F = A halves that stream at 4 and 8 GPUs (2A2F, 4A4F), where 3A1F /
# 6A2F would leave one or two FFN ranks reading 64 / 32 experts per layer.
TOPOLOGY = {1: (0, 0), 2: (1, 1), 4: (2, 2), 8: (4, 4)}
MODEL_DESC = {
    "deepseek-v2-lite": "DeepSeek-V2-Lite (27 layers, 64 experts top-6, MLA 16 heads)",
    "qwen3-30b-a3b": "Qwen3-30B-A3B (48 layers, 128 experts top-8, GQA 32q/4kv)",
    "deepseek-v3-32l": "DeepSeek-V3 shapes truncated to 32 layers (fp8 block-scaled experts)",
}


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="deepseek-v2-lite")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--isl", type=int, default=1024)
    ap.add_argument("--osl", type=int, default=256)
    ap.add_argument("--connector", default="auto", choices=["auto", "b200", "nccl"])
    ap.add_argument("--eager", action="store_true", help="disable CUDA graphs")
    ap.add_argument("--dbo", action="store_true",
                    help="two-ubatch dual-batch overlap (off by default: the FFN step is weight-bandwidth bound, "
                         "so a second ubatch re-reads every expert weight)")
    ap.add_argument("--no-dbo", action="store_true", help="force DBO off")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sync-scheduling", action="store_true",
                    help="end-to-end loop: read each step's tokens before launching the next (the default "
                         "launches step t+1 before reading step t back, EngineConfig.async_scheduling)")
    ap.add_argument("--layers", type=int, default=0,
                    help="truncate the model to this many layers for quick checks; the line is marked invalid")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip counting this package's kernels per step (the count runs one eager step under "
                         "torch.profiler, which conflicts with an outside profiler such as ncu)")
    ap.add_argument("--topology", default="", help="override A,F split for N>1, e.g. 4,4 or 2,2")
    ap.add_argument("--phases", action="store_true",
                    help="diagnostic: per-role phase timing on the device (adds a stamp kernel per phase)")
    return ap.parse_args(argv)


# ---------------------------------------------------------------- reference
def reference_arm(args) -> None:
    """The unmodified reference (``baseline/_ref``) on its stock path: ``bench_reference.py``."""
    import bench_reference

    bench_reference.main(args, METRIC, MODEL_DESC.get(args.model, args.model))


# ------------------------------------------------------------------ helpers
def build_config(args, *, num_attn: int, num_ffn: int, role: str | None, connector: str):
    from afd_plugin_b200.engine_config import CacheConfig, CompilationConfig, EngineConfig, ModelConfig, ParallelConfig
    from afd_plugin_b200.models.configs import get_preset

    arch = get_preset(args.model)
    if args.layers:
        arch = arch.scaled(num_hidden_layers=args.layers)
    per_rank = math.ceil(args.batch / max(1, num_attn))
    additional = {}
    if role is not None:
        additional["afd"] = {"role": role, "connector": connector, "num_attention_ranks": num_attn,
                             "num_ffn_ranks": num_ffn, "compute_gate_on_attention": False}
    max_len = args.isl + args.osl
    return EngineConfig(
        model_config=ModelConfig(arch, dtype=torch.bfloat16, enforce_eager=args.eager, max_model_len=max_len + 64),
        parallel_config=ParallelConfig(data_parallel_size=max(1, num_attn), use_ubatching=args.dbo,
                                       num_ubatches=2 if args.dbo else 1),
        compilation_config=CompilationConfig(cudagraph_capture_sizes=[per_rank]),
        cache_config=CacheConfig(block_size=64),
        additional_config=additional,
        max_num_seqs=per_rank,
        async_scheduling=not args.sync_scheduling,
    ), per_rank


def count_our_kernels(fn) -> int:
    """Number of this package's kernels one call of ``fn`` launches (profiler count, untimed)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "afd::" in e.name)


def one_eager_step(engine, batch: int) -> None:
    from afd_plugin_b200.runtime.model_runner import ubatch_splits

    engine.runner._decode_body(batch, ubatch_splits(batch, engine.runner.num_ubatches))
    engine.runner.advance_on_device(batch)


def prime_requests(engine, n: int, isl: int, osl: int, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    vocab = engine.model.arch.vocab_size
    prompts = torch.randint(0, vocab, (n, isl), generator=g).tolist()
    first = torch.randint(0, vocab, (n,), generator=g).tolist()
    engine.admit_prefilled(prompts, first, reserve_tokens=osl)
    engine.kv.fill_random_(seed=seed, std=1.0)


def device_loop(engine, batch: int, warmup: int, steps: int, isl: int, osl: int, barrier=None):
    """Graph replay + on-device advance; returns per-step ms list (events).

    ``barrier`` (multi-rank) brackets the timed region together with a device
    synchronize on both sides.
    """
    runner = engine.runner
    use_graph = batch in runner.graphs
    wrap_at, wrap_to = isl + osl - 1, isl

    def one():
        runner.decode_step(batch, use_graph=use_graph)
        runner.advance_on_device(batch, wrap_at=wrap_at, wrap_to=wrap_to)

    engine.load_decode_batch()
    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    if barrier is not None:
        barrier()
    nvtx = os.environ.get("AFD_BENCH_NVTX") == "1"
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    if nvtx:
        torch.cuda.nvtx.range_push("timed")
    ev[0].record()
    for i in range(steps):
        one()
        ev[i + 1].record()
    torch.cuda.synchronize()
    if barrier is not None:
        barrier()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    return [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)], ev[0].elapsed_time(ev[-1])


def e2e_loop(engine, warmup: int, steps: int):
    """Public-API steps: H2D of inputs, replay, D2H of tokens each step."""
    for _ in range(warmup):
        engine.step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        engine.step()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) * 1e3, engine.last_h2d_bytes, engine.last_d2h_bytes


def _log(msg: str) -> None:
    if os.environ.get("AFD_BENCH_VERBOSE") == "1":
        print(f"[rank {os.environ.get('RANK', '0')}] {msg}", file=sys.stderr, flush=True)


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        reference_arm(args)
        return 0
    if args.phases:
        os.environ["AFD_PHASE_TIMING"] = "1"
    from afd_plugin_b200.utils.clocks import ClockSampler

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if args.gpus not in TOPOLOGY:
        raise SystemExit(f"unsupported --gpus {args.gpus}; use 1, 2, 4 or 8")
    num_attn, num_ffn = TOPOLOGY[args.gpus]
    if args.no_dbo:
        args.dbo = False
    if args.topology:
        num_attn, num_ffn = (int(x) for x in args.topology.split(","))
        if num_attn + num_ffn != args.gpus:
            raise SystemExit("--topology A,F must add up to --gpus")
    connector = {"auto": "P2pNcclAFDConnector", "nccl": "P2pNcclAFDConnector",
                 "b200": "B200FusedAFDConnector"}[args.connector]
    if args.connector == "auto":
        try:
            from afd_plugin_b200.connectors import b200_fused  # noqa: F401

            connector = "B200FusedAFDConnector"
        except ImportError:
            pass
    result: dict = {}
    if args.gpus == 1:
        from afd_plugin_b200.models import build_model
        from afd_plugin_b200.runtime.engine import LLMEngine

        ec, per_rank = build_config(args, num_attn=0, num_ffn=0, role=None, connector=connector)
        model = build_model(ec.model_config.arch, role="colocated", dtype=torch.bfloat16, device="cuda", seed=0,
                            max_positions=ec.model_config.max_model_len)
        engine = LLMEngine(ec, model)
        prime_requests(engine, args.batch, args.isl, args.osl)
        if not args.eager:
            engine.capture_graphs()
        batch = len(engine.running)
        engine.load_decode_batch()
        launches_per_step = 0 if args.no_launch_count else count_our_kernels(lambda: one_eager_step(engine, batch))
        with ClockSampler(local) as clk:
            per_step, total_ms = device_loop(engine, batch, args.warmup, args.steps, args.isl, args.osl)
            e2e = None
            if not args.no_e2e:
                e2e_ms, h2d, d2h = e2e_loop(engine, args.warmup, args.steps)
                e2e = {"value": round(batch * args.steps / (e2e_ms / 1e3), 1), "unit": "tok/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        result = dict(ms=total_ms, per_step=per_step, tokens=batch, e2e=e2e, clocks=clk.summary(),
                      launches=launches_per_step * args.steps, parallelism="colocated-1gpu",
                      phases=[{"rank": 0, "role": "colocated", "phases": engine.runner.timer.summary()}])
        status = torch.ops.afd_b200.read_status(local)
        if status:
            raise RuntimeError(f"kernel status word {status} (a bounded wait expired)")
        engine.runner.release_graphs()
    else:
        from afd_plugin_b200.bench.afd_decode import run_afd_rank

        result = run_afd_rank(args, rank=rank, local=local, num_attn=num_attn, num_ffn=num_ffn, connector=connector,
                              build_config=build_config, prime_requests=prime_requests, device_loop=device_loop,
                              e2e_loop=e2e_loop, count_our_kernels=count_our_kernels, log=_log)
    if rank == 0:
        ms = result["ms"]
        tokens_per_step = args.batch
        value = tokens_per_step * args.steps / (ms / 1e3)
        clocks = result.get("clocks") or {}
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "tok/s",
            "n_gpus": args.gpus,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "p50_tpot_ms": round(statistics.median(result["per_step"]), 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
            "dtype": "bf16",
            "data": "synthetic (random-init weights; random prompt ids with synthetic prompt KV, decode only)",
            "config": {
                "model": MODEL_DESC.get(args.model, args.model),
                "global_batch": args.batch,
                "seq_len": args.isl + args.osl,
                "input_len": args.isl,
                "output_len": args.osl,
                "parallelism": result["parallelism"],
                "cuda_graphs": not args.eager,
                "dbo": args.dbo,
                "e2e_scheduling": "sync" if args.sync_scheduling else "async",
                "l2": "inputs larger than L2 (31 GB weights, ~10 GB KV per step); no flush",
            },
            "clocks": {"sm_mhz": clocks.get("sm_mhz"), "sm_max_mhz": clocks.get("sm_max_mhz"),
                       "reasons": clocks.get("reasons", [])},
            "e2e": result.get("e2e"),
            "gpu_launches": result.get("launches"),
        }
        if args.layers:
            line["invalid_as_bench"] = f"model truncated to {args.layers} layers"
        if args.phases:
            line["phases"] = result.get("phases")
            line["note"] = "phase-timing run: stamp kernels inside the step; a diagnostic, not a bench value"
        print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
