"""Paged MLA decode kernel at decode-step shapes: device time and KV bandwidth.

Decode attention reads every cached latent row once per step (576 bf16 = 1152
bytes per token and layer); the figure of merit is those bytes per second
against the measured HBM copy bandwidth (``MEASURED_PEAKS.json`` at the
repository root, when present).  Each timed launch follows a 256 MiB read
that evicts L2 (126 MB), so the cache is read from HBM at every shape.

    python -m afd_plugin_b200.bench.mla_decode_bench [--shapes dsv2-lite-b256,...] [--reps 3]
    python -m afd_plugin_b200.bench.mla_decode_bench --sparse

``--sparse`` compares DeepSeek-sparse-attention decode (the indexer's kept
positions) on the sm_100a gather kernel against the gather + two batched
GEMMs of ``ops/reference.py::mla_decode_sparse``.  The kernel is chosen per
process by the environment: ``AFD_MLA_KERNEL=mma`` (the mma.sync split
kernel at every head count), ``AFD_MLA_BALANCED=1`` (the work-balanced
kernel for 16-head groups), ``AFD_MLA_TC_SHAPE`` (a tcgen05 shape).
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from afd_plugin_b200.bench.grouped_gemm_bench import _peak_gbs

# name: (batch, heads, context tokens)
SHAPES = {
    "dsv2-lite-b256": (256, 16, 1034),   # the 1-GPU decode step: 256 requests, ~1 K context
    "dsv2-lite-b64": (64, 16, 1034),     # one Attention rank of 4A4F (8 GPUs)
    "dsv2-lite-b43": (43, 16, 1034),     # one Attention rank of 6A2F
    "dsv3-b64": (64, 128, 2100),         # DeepSeek-V3 heads, one Attention rank of 4A4F
}


def run(shape: str, reps: int, bs: int = 64, splits: int = 0) -> dict:
    from afd_plugin_b200.ops import _ext

    C = _ext.ops()
    B, H, ctx = SHAPES[shape]
    dev = "cuda"
    nblk = math.ceil(ctx / bs)
    cache = torch.randn(B * nblk + 1, bs, 576, device=dev, dtype=torch.bfloat16)
    table = (torch.randperm(B * nblk, device=dev).view(B, nblk) + 1).to(torch.int32)
    seq = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, H, 576, device=dev, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(192)
    fn = lambda: C.mla_decode(q[..., :512], q[..., 512:], cache, table, seq, scale, splits, False)  # noqa: E731
    med = _median_us(fn, reps)
    kv_bytes = B * ctx * 576 * 2
    peak, kind = _peak_gbs()
    gbs = kv_bytes / (med * 1e-6) / 1e9
    return {"shape": shape, "batch": B, "heads": H, "context": ctx, "splits": splits or "auto", "us_median": round(med, 2),
            "kv_GBps": round(gbs, 1), f"frac_of_{kind}_hbm": round(gbs / peak, 3),
            "status": int(C.read_status(torch.cuda.current_device()))}


# name: (batch, heads, context tokens, kept positions)
SPARSE = {
    "dsv32-b64-8k": (64, 128, 8192, 2048),   # DeepSeek-V3.2 heads and index_topk, one Attention rank
    "dsv32-b16-32k": (16, 128, 32768, 2048),
    "dsv32-b256-4k-h16": (256, 16, 4096, 2048),
}


_FLUSH = None


def _median_us(fn, reps: int) -> float:
    """Median device time of ``fn`` over ``reps`` launches, each after a
    256 MiB read that evicts the 126 MB L2 (the KV of the smaller shapes
    would otherwise stay cached between launches).  A read leaves clean lines,
    as the weight-reading kernels before attention do in a decode step; a
    write would leave dirty lines whose write-back the timed kernel would pay."""
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    start = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    end = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    for i in range(reps):
        _FLUSH.sum()
        start[i].record()
        fn()
        end[i].record()
    torch.cuda.synchronize()
    us = sorted(start[i].elapsed_time(end[i]) * 1e3 for i in range(reps))
    return us[len(us) // 2]


def run_sparse(shape: str, reps: int, bs: int = 64) -> dict:
    from afd_plugin_b200.ops import _ext
    from afd_plugin_b200.ops import reference as ref

    C = _ext.ops()
    B, H, ctx, K = SPARSE[shape]
    dev = "cuda"
    nblk = math.ceil(ctx / bs)
    cache = torch.randn(B * nblk + 1, bs, 576, device=dev, dtype=torch.bfloat16)
    table = (torch.randperm(B * nblk, device=dev).view(B, nblk) + 1).to(torch.int32)
    seq = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    keep = torch.stack([torch.randperm(ctx, device=dev)[:K] for _ in range(B)]).to(torch.int32)
    q = torch.randn(B, H, 576, device=dev, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(192)
    kern = lambda: C.mla_decode_sparse(q, cache, table, seq, keep, scale, 0)  # noqa: E731
    gath = lambda: ref.mla_decode_sparse(q, cache, table, keep, scale, 512)  # noqa: E731
    got, want = kern().float(), gath().float()
    err = float((got - want).abs().max() / (want.abs().max() + 1e-6))
    return {"shape": shape, "batch": B, "heads": H, "context": ctx, "kept": K,
            "kernel_us": round(_median_us(kern, reps), 2), "gather_bmm_us": round(_median_us(gath, reps), 2),
            "max_rel_diff": round(err, 4), "status": int(C.read_status(torch.cuda.current_device()))}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--splits", default="0", help="comma list of KV split counts (0 = the kernel's own pick)")
    ap.add_argument("--sparse", action="store_true", help="sparse (indexer-selected) decode: kernel vs gather + bmm")
    args = ap.parse_args(argv)
    if args.sparse:
        for shape in SPARSE:
            print(json.dumps(run_sparse(shape, args.reps)), flush=True)
        return
    for shape in args.shapes.split(","):
        for sp in args.splits.split(","):
            print(json.dumps(run(shape, args.reps, splits=int(sp))), flush=True)


if __name__ == "__main__":
    main()
