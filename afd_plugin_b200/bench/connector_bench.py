"""Connector microbenchmark: dispatch + combine round trip, fused vs NCCL.

    torchrun --nproc-per-node A+F -m afd_plugin_b200.bench.connector_bench \
        --attn A --ffn F [--tokens 1,2,4,...,1024] [--hidden 7168 --experts 256 --topk 8]

Payload (the reference's connector sweep: DeepSeek-V3 width): hidden-7168 bf16 rows, top-8 routing over 256
experts from N(0, 1) logits with softmax weights.

* ``fused``: Attention ranks run the fused dispatch kernel (norm, router,
  top-k, one row per destination FFN rank + routing); FFN ranks run the
  combine-send kernel in transport-only mode (each received row scaled by its
  local routing weights and stored back into the source's slot, i.e. the
  expert GEMMs replaced by identity) and the Attention ranks run
  ``afd_combine``.  Bytes over NVLink per token: one row per destination FFN
  rank each way (+ 8 bytes per routed expert of routing metadata).
* ``nccl``: the reference wire protocol -- each Attention rank sends its
  ``[T, H]`` hidden states to its FFN rank and receives ``[T, H]`` back
  (NCCL send/recv on the FFN subgroup's communicator, stream-ordered as the
  NCCL connector issues them).  Bytes per token: one row each way.

Both paths are timed as the decode step runs them: ``--iters`` round trips
captured into one CUDA graph per rank, replayed after a barrier, CUDA-event
timed per rank; the max over ranks is reported (``--eager`` times plain
launches instead), with the achieved GB/s (bytes one Attention rank moves out
and in) and the fraction of the NVLink roofline (measured 770 GB/s per
direction per GPU).
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

NVLINK_GBPS = 770.0


def _args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--attn", type=int, default=1)
    ap.add_argument("--ffn", type=int, default=1)
    ap.add_argument("--tokens", default="1,2,4,8,16,32,64,128,256,512,1024")
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--paths", default="fused,nccl")
    ap.add_argument("--out", default="")
    ap.add_argument("--fp8", action="store_true", help="rows travel as e4m3 with 1x128 scales (fused path)")
    ap.add_argument("--eager", action="store_true", help="time plain launches instead of a CUDA graph replay")
    ap.add_argument("--wait-timeout-ms", type=int, default=2000,
                    help="bound of every in-kernel wait of the fused path (a missed flag ends the wait with an error)")
    ap.add_argument("--breakdown", action="store_true",
                    help="time each kernel of single round trips (barrier between trips)")
    return ap.parse_args(argv)


def _timed_us(fn, args) -> float:
    """Device time per call of ``fn`` on this rank: ``args.iters`` calls
    captured into one CUDA graph (or launched eagerly with ``--eager``),
    every rank starting after a barrier."""
    dist.barrier()
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.eager:
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        return e0.elapsed_time(e1) * 1e3 / args.iters
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(args.iters):
            fn()
    torch.cuda.synchronize()
    dist.barrier()
    graph.replay()  # warm replay
    torch.cuda.synchronize()
    dist.barrier()
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    del graph  # released before any communicator it recorded is destroyed
    return e0.elapsed_time(e1) * 1e3 / args.iters


def _max_over_ranks(x: float) -> float:
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def bench_fused(args, rank: int, tokens: list[int]) -> list[dict]:
    from afd_plugin_b200.config import afd_config_from_mapping
    from afd_plugin_b200.connectors.b200_fused import B200FusedAFDConnector
    from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
    from afd_plugin_b200.models.configs import DSV3_32L
    from afd_plugin_b200.parallel.topology import role_of_world_rank

    A, F = args.attn, args.ffn
    role, role_rank = role_of_world_rank(rank, attention_size=A, ffn_size=F)
    arch = DSV3_32L.scaled(hidden_size=args.hidden, n_routed_experts=args.experts, num_experts_per_tok=args.topk,
                           num_hidden_layers=1, quant=None, scoring_func="softmax", topk_method="greedy",
                           n_shared_experts=0, routed_scaling_factor=1.0, norm_topk_prob=False)
    t_cap = max(tokens)
    afd = afd_config_from_mapping({
        "role": role, "connector": "B200FusedAFDConnector", "num_attention_ranks": A, "num_ffn_ranks": F,
        "connector_extra_config": {"max_tokens_per_rank": t_cap, "expert_capacity_factor": 4.0,
                                   "fp8_dispatch": bool(args.fp8),
                                   "wait_timeout_ms": args.wait_timeout_ms}})
    ec = EngineConfig(ModelConfig(arch, dtype=torch.bfloat16), additional_config={"afd": {}}, max_num_seqs=t_cap)
    conn = B200FusedAFDConnector(rank, rank, ec, afd, role_rank)
    conn.init_afd_connector()
    C = torch.ops.afd_b200
    d = conn.dims
    H = args.hidden
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    gate_w = (torch.randn(args.experts, H, device="cuda", generator=g) / H ** 0.5).to(torch.bfloat16)
    norm_w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    results = []
    for T in tokens:
        x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
        res = torch.zeros_like(x)

        def step_attn():
            C.afd_epoch(conn.epoch[0:1])
            r = res.clone()
            cfg = [args.experts, args.topk, 0, 0, 1, 1, 1, 0, F, d.e_local, d.t_cap, role_rank,
                   role_rank // d.ratio, 0]
            C.afd_dispatch(x, r, norm_w, 1e-6, gate_w, None, 1.0, conn.dispatch_ptrs[0], conn.fmask[0],
                           conn.dctr[0], cfg)
            return C.afd_combine(conn.comb[0], conn.fmask[0], T, conn.comb_flag[0], 0, conn.epoch[0:1], F,
                                 conn.timeout_ns)

        def step_ffn():
            C.afd_epoch(conn.epoch[0:1])
            C.afd_wait(conn.arrive[0], 0, conn.epoch[0:1], A, conn.timeout_ns)
            C.afd_combine_send(conn.tok[0], conn.rid[0], conn.rwt[0], conn.tcount[0], conn.comb_ptrs[0],
                               conn.comb_flag_ptrs[0], conn.done[0, 2:3], H,
                               [A, d.t_cap, args.topk, d.slots, d.e_local, role_rank * d.e_local, d.ratio,
                                role_rank * d.ratio, 1, 0, role_rank, F, 0, 1],
                               tok_scale=conn.tok_scale[0] if conn.dims.fp8 else None)

        fn = step_attn if role == "attention" else step_ffn
        if args.breakdown:
            results.append(_breakdown(args, role, T, conn, x, res, norm_w, gate_w, role_rank, d, A, F, H))
            continue
        us = _max_over_ranks(_timed_us(fn, args))
        status = int(C.read_status(torch.cuda.current_device()))
        # Rows this rank moved: one per (token, destination FFN rank) each way.
        if role == "attention":
            masks = conn.fmask[0, :T].cpu()
            dest = sum(bin(int(m)).count("1") for m in masks)
        else:
            dest = 0
        dest = int(_max_over_ranks(float(dest)))
        out_row = H + H // 32 if args.fp8 else 2 * H  # e4m3 row + fp32 scale per 128 columns, or bf16
        bytes_per_attn = dest * (out_row + 2 * H) + 2 * T * args.topk * 8 * F  # rows out + back, routing metadata
        gbps = bytes_per_attn / (us * 1e-6) / 1e9
        # roofline: each direction limited by one GPU's NVLink; the busiest GPU is an FFN rank
        # receiving from its share of the Attention ranks.
        ffn_rows = dest * A / F
        ideal_us = max(dest, ffn_rows) * max(out_row, 2 * H) / (NVLINK_GBPS * 1e9) * 1e6
        results.append({"path": "fused-fp8" if args.fp8 else "fused", "tokens": T, "us": round(us, 2),
                        "GBps": round(gbps, 1),
                        "rows_per_token": round(dest / max(1, T), 2),
                        "roofline_frac": round(ideal_us / us, 3), "status": status})
    conn.close()
    return results


def _breakdown(args, role, T, conn, x, res, norm_w, gate_w, role_rank, d, A, F, H) -> dict:
    """Median per-kernel device time over single round trips (both sides aligned by a barrier)."""
    import statistics

    C = torch.ops.afd_b200
    names = ["epoch", "dispatch", "combine"] if role == "attention" else ["epoch", "wait", "combine_send"]
    rows = {n: [] for n in names}
    for it in range(args.warmup + args.iters):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        torch.cuda.synchronize()
        dist.barrier()
        ev[0].record()
        C.afd_epoch(conn.epoch[0:1])
        ev[1].record()
        if role == "attention":
            r = res.clone()
            cfg = [args.experts, args.topk, 0, 0, 1, 1, 1, 0, F, d.e_local, d.t_cap, role_rank, role_rank // d.ratio, 0]
            C.afd_dispatch(x, r, norm_w, 1e-6, gate_w, None, 1.0, conn.dispatch_ptrs[0], conn.fmask[0],
                           conn.dctr[0], cfg)
            ev[2].record()
            C.afd_combine(conn.comb[0], conn.fmask[0], T, conn.comb_flag[0], 0, conn.epoch[0:1], F, conn.timeout_ns)
        else:
            C.afd_wait(conn.arrive[0], 0, conn.epoch[0:1], A, conn.timeout_ns)
            ev[2].record()
            C.afd_combine_send(conn.tok[0], conn.rid[0], conn.rwt[0], conn.tcount[0], conn.comb_ptrs[0],
                               conn.comb_flag_ptrs[0], conn.done[0, 2:3], H,
                               [A, d.t_cap, args.topk, d.slots, d.e_local, role_rank * d.e_local, d.ratio,
                                role_rank * d.ratio, 1, 0, role_rank, F, 0, 1],
                               tok_scale=conn.tok_scale[0] if conn.dims.fp8 else None)
        ev[3].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            for i, n in enumerate(names):
                rows[n].append(ev[i].elapsed_time(ev[i + 1]) * 1e3)
    out = {"path": "fused-breakdown", "tokens": T}
    for n in names:
        out[n + "_us"] = round(statistics.median(rows[n]), 2)
    gathered = [None] * dist.get_world_size()
    dist.all_gather_object(gathered, out)
    merged = {"path": "fused-breakdown", "tokens": T}
    for g in gathered:
        merged.update({k: v for k, v in g.items() if k.endswith("_us")})
    return merged


def bench_nccl(args, rank: int, tokens: list[int]) -> list[dict]:
    from afd_plugin_b200.config import afd_config_from_mapping
    from afd_plugin_b200.parallel.topology import build_rank_mapping, role_of_world_rank

    from afd_plugin_b200.connectors.p2p_nccl import init_subgroup_comm
    from afd_plugin_b200.ops._ext import ops

    A, F = args.attn, args.ffn
    role, role_rank = role_of_world_rank(rank, attention_size=A, ffn_size=F)
    m = build_rank_mapping(afd_config_from_mapping({"role": role, "num_attention_ranks": A, "num_ffn_ranks": F}),
                           role_rank)
    comm = init_subgroup_comm(m, attention_size=A, ffn_size=F, device=torch.device("cuda", torch.cuda.current_device()))
    send, recv = torch.ops.afd_b200.nccl_send, torch.ops.afd_b200.nccl_recv
    H = args.hidden
    results = []
    for T in tokens:
        if role == "attention":  # subgroup rank 0 is the FFN rank
            x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
            y = torch.empty_like(x)

            def fn():
                send(x, 0, comm)
                recv(y, 0, comm)
        else:  # subgroup ranks 1..A/F are this FFN rank's Attention ranks
            bufs = [torch.empty(T, H, device="cuda", dtype=torch.bfloat16) for _ in range(A // F)]

            def fn():
                for j, b in enumerate(bufs):
                    recv(b, j + 1, comm)
                for j, b in enumerate(bufs):
                    send(b, j + 1, comm)

        us = _max_over_ranks(_timed_us(fn, args))
        bytes_per_attn = 2 * T * H * 2
        gbps = bytes_per_attn / (us * 1e-6) / 1e9
        ideal_us = (T * H * 2 * (A // F)) / (NVLINK_GBPS * 1e9) * 1e6  # the FFN rank serves A/F peers
        results.append({"path": "nccl", "tokens": T, "us": round(us, 2), "GBps": round(gbps, 1),
                        "roofline_frac": round(ideal_us / us, 3)})
    torch.cuda.synchronize()
    ops().nccl_comm_destroy(comm)
    return results


def main(argv=None) -> int:
    args = _args(argv)
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    if dist.get_world_size() != args.attn + args.ffn:
        raise SystemExit("world size must equal --attn + --ffn")
    tokens = [int(t) for t in args.tokens.split(",")]
    rows = []
    for path in args.paths.split(","):
        rows += bench_fused(args, rank, tokens) if path == "fused" else bench_nccl(args, rank, tokens)
    if rank == 0:
        topo = f"{args.attn}A{args.ffn}F"
        for r in rows:
            r["topology"] = topo
            print(json.dumps(r))
        if args.out:
            with open(args.out, "a") as fh:
                for r in rows:
                    fh.write(json.dumps(r) + "\n")
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
