"""Multi-GPU AFD decode benchmark body (one process per GPU, torchrun).

Attention ranks run the device-resident decode loop and then the public-API
loop; FFN ranks serve exactly the steps the Attention side issues.  Every
rank times its own loop with CUDA events; the reported time is the max over
ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from afd_plugin_b200.parallel.topology import role_of_world_rank
from afd_plugin_b200.utils.clocks import ClockSampler


def run_afd_rank(args, *, rank, local, num_attn, num_ffn, connector, build_config, prime_requests, device_loop,
                 e2e_loop, count_our_kernels, log=lambda msg: None) -> dict:
    from datetime import timedelta

    # Lazy NCCL init: with an eagerly bound device, new_group() becomes a
    # communicator split that every rank must enter before any other traffic.
    dist.init_process_group("nccl", timeout=timedelta(seconds=180))
    log("process group up")
    role, role_rank = role_of_world_rank(rank, attention_size=num_attn, ffn_size=num_ffn)
    ec, per_rank = build_config(args, num_attn=num_attn, num_ffn=num_ffn, role=role, connector=connector)
    # Even split of the global batch over the Attention ranks.
    shares = [args.batch // num_attn + (1 if i < args.batch % num_attn else 0) for i in range(num_attn)]
    total_steps = 2 * (args.warmup + args.steps) + (0 if args.no_e2e else 0)
    result: dict = {"parallelism": f"afd-{num_attn}A{num_ffn}F-{connector}"}
    if role == "ffn":
        from afd_plugin_b200.runtime.workers import AFDFFNWorker

        w = AFDFFNWorker(ec, local_rank=local)
        w.model_runner.count_next_eager = True
        log("ffn worker ready, serving")
        # Serve right away: the Attention side's warmup and graph capture already
        # send control payloads.  The loop ends on the shutdown payload.
        with ClockSampler(local) as clk:
            n = w.run_ffn_server_loop()
        result.update(ms=0.0, per_step=[0.0], clocks=clk.summary(), steps_served=n,
                      launches_local=w.model_runner.kernels_per_step * args.steps,
                      phases=getattr(getattr(w.model_runner, "timer", None), "summary", dict)())
        w.shutdown()
    else:
        from afd_plugin_b200.runtime.workers import AFDAttentionWorker

        w = AFDAttentionWorker(ec, local_rank=local)
        log("attention worker ready")
        eng = w.engine
        prime_requests(eng, shares[role_rank], args.isl, args.osl, seed=role_rank)
        log("requests primed")
        from bench import one_eager_step  # the same decode step the timed loop runs

        per_step_kernels = count_our_kernels(lambda: one_eager_step(eng, len(eng.running)))
        if not args.eager:
            eng.capture_graphs()
            log("graphs captured")
        batch = len(eng.running)
        grp = w.groups.attention_group
        barrier = (lambda: dist.barrier(group=grp)) if num_attn > 1 else None
        with ClockSampler(local) as clk:
            per_step, ms = device_loop(eng, batch, args.warmup, args.steps, args.isl, args.osl, barrier=barrier)
            e2e = None
            if not args.no_e2e:
                e2e_ms, h2d, d2h = e2e_loop(eng, args.warmup, args.steps)
                e2e = (e2e_ms, h2d, d2h)
        result.update(ms=ms, per_step=per_step, clocks=clk.summary(), e2e_raw=e2e, batch=batch,
                      launches_local=per_step_kernels * args.steps, phases=eng.runner.timer.summary())
        log("timed loops done")
        if barrier is not None:
            barrier()
        w.shutdown()
    # Max over ranks of the device-timed loop, its p50 step and the e2e wall time;
    # sums of launches and host<->device bytes.
    import statistics

    p50 = statistics.median(result["per_step"]) if role == "attention" else 0.0
    e2e_ms, h2d, d2h = result.get("e2e_raw") or (0.0, 0, 0)
    mx = torch.tensor([result["ms"], e2e_ms, p50], dtype=torch.float64, device="cuda")
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    sm = torch.tensor([float(result.get("launches_local", 0)), float(h2d), float(d2h)], dtype=torch.float64,
                      device="cuda")
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    result["ms"] = float(mx[0])
    result["per_step"] = [float(mx[2])]
    if not args.no_e2e and float(mx[1]) > 0:
        result["e2e"] = {"value": round(args.batch * args.steps / (float(mx[1]) / 1e3), 1), "unit": "tok/s",
                         "h2d_bytes_per_step": int(sm[1]), "d2h_bytes_per_step": int(sm[2])}
    result["launches"] = int(sm[0])
    if args.phases:
        every = [None] * dist.get_world_size()
        dist.all_gather_object(every, {"rank": rank, "role": role, "role_rank": role_rank,
                                       "phases": result.get("phases", {})})
        result["phases"] = every
    dist.barrier()
    dist.destroy_process_group()
    return result


__all__ = ["run_afd_rank"]
