"""Kernel timeline of one colocated decode step (the bench configuration on one GPU).

Builds the `bench.py` engine (DeepSeek-V2-Lite shapes, random weights,
synthetic prompt KV), captures the decode graph, times ``--steps`` replays
with CUDA events, then records three more replays under ``torch.profiler``
(CUDA activity) and prints, for the middle one: the step's span, each kernel
name's total time, count and summed gap before it, and the kernel sequence of
one decoder layer.  The profiler run is for the shares and the sequence; the
CUDA-event time printed first is the step time.

    python -m afd_plugin_b200.bench.step_timeline [--batch 64] [--layer 5] [--json out.json]
"""

from __future__ import annotations

import argparse
import collections
import json
import os
import sys

import torch


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--model", default="deepseek-v2-lite")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--layer", type=int, default=5, help="decoder layer whose kernel sequence is listed")
    ap.add_argument("--json", default="", help="also write every recorded kernel (name, start, end) here")
    args = ap.parse_args(argv)

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    if root not in sys.path:
        sys.path.insert(0, root)
    import bench
    from torch.profiler import ProfilerActivity, profile

    from afd_plugin_b200.models import build_model
    from afd_plugin_b200.runtime.engine import LLMEngine

    bargs = bench.parse_args(["--batch", str(args.batch), "--model", args.model])
    ec, _ = bench.build_config(bargs, num_attn=0, num_ffn=0, role=None, connector="colocated")
    model = build_model(ec.model_config.arch, role="colocated", dtype=torch.bfloat16, device="cuda", seed=0,
                        max_positions=ec.model_config.max_model_len)
    engine = LLMEngine(ec, model)
    bench.prime_requests(engine, bargs.batch, bargs.isl, bargs.osl)
    engine.capture_graphs()
    batch = len(engine.running)
    _, total_ms = bench.device_loop(engine, batch, 5, args.steps, bargs.isl, bargs.osl)
    print(f"decode step: {total_ms / args.steps:.3f} ms (CUDA events, {args.steps} graph replays)")

    runner = engine.runner
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(3):
            runner.decode_step(batch, use_graph=True)
            runner.advance_on_device(batch, wrap_at=bargs.isl + bargs.osl - 1, wrap_to=bargs.isl)
        torch.cuda.synchronize()
    evs = sorted((e for e in prof.events() if e.device_type.name == "CUDA"), key=lambda e: e.time_range.start)
    rows = [(e.name, e.time_range.start, e.time_range.end) for e in evs]
    if args.json:
        with open(args.json, "w") as fh:
            json.dump(rows, fh)
    n = len(rows) // 3
    step = rows[n : 2 * n]
    print(f"profiled step: {step[-1][2] - step[0][1]:.1f} us span, {len(step)} kernels")
    agg: dict = collections.OrderedDict()
    prev = None
    for name, s, e in step:
        d = agg.setdefault(name[:100], [0, 0.0, 0.0])
        d[0] += 1
        d[1] += e - s
        if prev is not None:
            d[2] += s - prev
        prev = e
    print(f"{'us':>9} {'count':>5} {'gap us':>8}  kernel")
    for k, (c, t, g) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        print(f"{t:9.1f} {c:5d} {g:8.1f}  {k}")
    marks = [i for i, r in enumerate(step) if "mla_decode" in r[0] or "gqa_decode" in r[0]]
    if len(marks) > args.layer + 1:
        lo, hi = marks[args.layer], marks[args.layer + 1]
        print(f"-- kernels from attention of layer {args.layer} to layer {args.layer + 1}")
        prev = None
        for name, s, e in step[lo : hi + 1]:
            print(f"  {e - s:7.1f} us  gap {0.0 if prev is None else s - prev:6.1f}  {name[:110]}")
            prev = e


if __name__ == "__main__":
    main()
