"""Grouped expert GEMM (tcgen05) at decode shapes: device time and weight bandwidth.

Decode MoE GEMMs are weight-streaming: every expert's weights are read once
per step while only a few tokens reuse them.  The figure of merit is the
weight bytes moved per second against the measured HBM copy bandwidth
(``MEASURED_PEAKS.json`` at the repository root, when present).

    python -m afd_plugin_b200.bench.grouped_gemm_bench [--shapes dsv2-lite-f2,...]
    python -m afd_plugin_b200.bench.grouped_gemm_bench --dense [--shapes in_proj,...]

``AFD_GG_PIPE=64|128|256`` selects the kernel's tokens per pass (and with it
the pipeline depth: 8, 6 or 4 stages) for a comparison run.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

# name: (local experts, hidden, intermediate, tokens per expert[, shared chunks, rows per shared chunk])
SHAPES = {
    "dsv2-lite-f2": (32, 2048, 1408, 24),     # DeepSeek-V2-Lite, 6A2F: 256 tokens x top-6 over 64 experts
    "dsv2-lite-f1": (64, 2048, 1408, 24),     # DeepSeek-V2-Lite, one FFN rank holds every expert
    # one GPU, 256-token decode batch: 64 routed experts plus the 2 shared-expert
    # chunks (virtual experts of the routed width) that see every token
    "dsv2-lite-colo": (64, 2048, 1408, 24, 2, 256),
    "qwen3-30b-f4": (32, 2048, 768, 32),      # Qwen3-30B-A3B, 4A4F: 512 tokens x top-8 over 128 experts
    "dsv3-f4": (64, 7168, 2048, 16),          # DeepSeek-V3 shapes, 4A4F: 512 tokens x top-8 over 256 experts
    "dsv3-e8": (8, 7168, 2048, 16),           # the same experts, 8 of them (profiling-sized, still > L2)
    "dsv3-e24": (24, 7168, 2048, 16),         # 24 of them: about five waves of (expert, tile) items
}


def _peak_gbs() -> tuple[float, str]:
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _time_us(fn, reps: int, iters: int = 5) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (iters * reps)


def _quant(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    from afd_plugin_b200.ops import reference as ref

    qs, ss = zip(*(ref.quant_fp8_block_weight(w[e]) for e in range(w.shape[0])))
    return torch.stack(qs).contiguous(), torch.stack(ss).contiguous()


def run(shape: str, reps: int, tokens_per_expert: int | None = None, fp8: bool = False) -> dict:
    from afd_plugin_b200.ops import _ext

    C = _ext.ops()
    E, H, I, tpe, *shared = SHAPES[shape]
    tpe = tokens_per_expert or tpe
    dev = "cuda"
    per = [tpe] * E + ([shared[1]] * shared[0] if shared else [])
    E = len(per)
    rows = sum(per)
    counts = torch.tensor(per, dtype=torch.int32, device=dev)
    offsets = torch.zeros(E, dtype=torch.int32, device=dev)
    offsets[1:] = counts.cumsum(0)[:-1]
    a1 = (torch.randn(rows, H, device=dev) * 0.1).to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=dev) * 0.02).to(torch.bfloat16)
    a2 = (torch.randn(rows, I, device=dev) * 0.1).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device=dev) * 0.02).to(torch.bfloat16)
    peak, kind = _peak_gbs()
    out = {"shape": shape, "experts": E, "hidden": H, "intermediate": I, "tokens_per_expert": tpe, "rows": rows,
           "weights": "fp8 e4m3, 128x128 block scales" if fp8 else "bf16"}
    if fp8:
        q13, s13 = _quant(w13)
        q2, s2 = _quant(w2)
        del w13, w2
        cases = (
            ("gemm1_swiglu", lambda: C.grouped_gemm_w8(a1, q13, s13, offsets, counts, 1, E), q13.numel() + s13.numel() * 4),
            ("gemm2", lambda: C.grouped_gemm_w8(a2, q2, s2, offsets, counts, 0, E), q2.numel() + s2.numel() * 4),
        )
    else:
        from afd_plugin_b200.ops.moe import moe_sync_buffer

        sync = moe_sync_buffer(torch.device(dev), E)
        cases = (
            ("gemm1_swiglu", lambda: C.grouped_gemm_ex(a1, w13, offsets, counts, 1, -1), w13.numel() * 2),
            ("gemm2", lambda: C.grouped_gemm_ex(a2, w2, offsets, counts, 0, -1), w2.numel() * 2),
            # both projections in one two-phase launch (what the MoE layers run)
            ("moe_ffn", lambda: C.moe_ffn(a1, w13, w2, offsets, counts, sync, max(per)),
             (w13.numel() + w2.numel()) * 2),
        )
    for name, fn, wbytes in cases:
        us = _time_us(fn, reps)
        gbs = wbytes / (us * 1e-6) / 1e9
        out[name + "_us"] = round(us, 2)
        out[name + "_weight_GBps"] = round(gbs, 1)
        out[name + f"_frac_of_{kind}_hbm"] = round(gbs / peak, 3)
    torch.cuda.synchronize()
    out["status"] = int(C.read_status(torch.cuda.current_device()))
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--tokens-per-expert", type=int, default=None)
    ap.add_argument("--fp8", action="store_true", help="fp8 block-scaled weights (grouped_gemm_w8)")
    args = ap.parse_args(argv)
    for shape in args.shapes.split(","):
        print(json.dumps(run(shape, args.reps, args.tokens_per_expert, fp8=args.fp8)), flush=True)




# Dense decode-step GEMMs of DeepSeek-V2-Lite at 256 tokens: (tokens, N, K, batch)
DENSE = {
    "in_proj": (256, 3712, 2048, 0),       # q + kv_a projections in one weight (rows padded to 128)
    "o_proj": (256, 2048, 2048, 0),
    "lm_head": (256, 102400, 2048, 0),
    "router": (256, 128, 2048, 0),         # 64 experts, rows padded to 128
    "w_uk": (256, 512, 128, 16),           # per head: q_nope [128] -> latent [512]
    "w_uv": (256, 128, 512, 16),           # per head: latent [512] -> v [128]
    "in_proj_b43": (43, 3712, 2048, 0),    # one Attention rank of 6A2F
    "o_proj_b43": (43, 2048, 2048, 0),
}


def run_dense(name: str, reps: int) -> dict:
    """tcgen05 ``tc_gemm`` vs torch (cuBLAS) on one dense or per-head batched shape."""
    from afd_plugin_b200.ops import _ext

    from afd_plugin_b200.ops.moe import gemm_workspace

    C = _ext.ops()
    ws = gemm_workspace(torch.device("cuda"))
    T, N, K, B = DENSE[name]
    dev = "cuda"
    if B:
        a = (torch.randn(B, T, K, device=dev) * 0.1).to(torch.bfloat16)
        w = (torch.randn(B, N, K, device=dev) * 0.02).to(torch.bfloat16)
        ours = lambda: C.tc_gemm(a, w, 0, 0, False, *ws)  # noqa: E731
        lib = lambda: torch.bmm(a, w.transpose(1, 2))  # noqa: E731
    else:
        a = (torch.randn(T, K, device=dev) * 0.1).to(torch.bfloat16)
        w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
        ours = lambda: C.tc_gemm(a, w, 0, 0, False, *ws)  # noqa: E731
        lib = lambda: torch.mm(a, w.t())  # noqa: E731
    wbytes = w.numel() * 2
    peak, kind = _peak_gbs()
    out = {"dense": name, "tokens": T, "n": N, "k": K, "batch": B}
    for tag, fn in (("tc_gemm", ours), ("cublas", lib)):
        us = _time_us(fn, reps)
        out[tag + "_us"] = round(us, 2)
        out[tag + f"_frac_of_{kind}_hbm"] = round(wbytes / (us * 1e-6) / 1e9 / peak, 3)
    return out


def main_dense(argv=None) -> None:
    ap = argparse.ArgumentParser(description="tcgen05 dense GEMMs vs cuBLAS at decode shapes")
    ap.add_argument("--shapes", default=",".join(DENSE))
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    for name in args.shapes.split(","):
        print(json.dumps(run_dense(name, args.reps)), flush=True)


if __name__ == "__main__":
    import sys

    if "--dense" in sys.argv:
        sys.argv.remove("--dense")
        main_dense()
    else:
        main()
