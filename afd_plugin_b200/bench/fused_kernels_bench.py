"""Device time of the fused AFD transfer kernels on one GPU (loopback).

The FFN ranks and the Attention rank are local buffers, so the row stores go
to local HBM instead of over NVLink: the numbers isolate the kernels' compute
and launch cost (norm, router, top-k, expand, slot sums) from the link.  Each
op is captured ``--reps`` times in one CUDA graph and timed with CUDA events.

    python -m afd_plugin_b200.bench.fused_kernels_bench [--tokens 1,43,256,1024]
"""

from __future__ import annotations

import argparse
import json

import torch

SHAPES = {  # name: (hidden, experts, top_k)
    "dsv2-lite": (2048, 64, 6),
    "qwen3-30b-a3b": (2048, 128, 8),
    "dsv3": (7168, 256, 8),
}


def _graph_time_us(fn, reps: int, iters: int = 5) -> float:
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


def run(shape: str, T: int, reps: int, F: int = 2) -> dict:
    from afd_plugin_b200.ops import _ext

    C = _ext.ops()
    H, E, k = SHAPES[shape]
    t_cap = max(T, 16)
    dev = "cuda"
    z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
    tok = [z(1, t_cap, H, dt=torch.bfloat16) for _ in range(F)]
    rid = [z(1, t_cap, k, dt=torch.int32) for _ in range(F)]
    rwt = [z(1, t_cap, k, dt=torch.float32) for _ in range(F)]
    tcount = [z(1, dt=torch.int32) for _ in range(F)]
    arrive = [z(1, dt=torch.int64) for _ in range(F)]
    ptrs = torch.tensor([[t.data_ptr() for t in grp] for grp in (tok, rid, rwt, tcount, arrive)],
                        dtype=torch.int64, device=dev)
    fmask = z(t_cap, dt=torch.int32)
    dctr = z(1 + (t_cap + 15) // 16, dt=torch.int32)
    x = torch.randn(T, H, device=dev).to(torch.bfloat16) * 0.01
    res = torch.randn(T, H, device=dev).to(torch.bfloat16)
    norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    gate = (torch.randn(E, H, device=dev) / H**0.5).to(torch.bfloat16)
    e_local = E // F
    cfg = [E, k, 0, 0, 1, 1, 1, 1, F, e_local, t_cap, 0, 0, 0]

    def dispatch():
        C.afd_dispatch(x, res, norm_w, 1e-6, gate, None, 1.0, ptrs, fmask, dctr, cfg)

    out = {"shape": shape, "tokens": T, "dispatch_us": round(_graph_time_us(dispatch, reps), 2)}

    cap = t_cap
    xs = z(e_local * cap, H, dt=torch.bfloat16)
    meta = z(e_local * cap, dt=torch.int32)
    rw = z(e_local * cap, dt=torch.float32)
    counts = z(e_local + 1, dt=torch.int32)

    def expand():
        counts.zero_()
        C.afd_expand(tok[0], rid[0], rwt[0], tcount[0], xs, meta, rw, counts, [1, t_cap, k, e_local, 0, cap, 1, 0, 1])

    out["expand_us"] = round(_graph_time_us(expand, reps), 2)
    comb = z(t_cap, F, H, dt=torch.bfloat16)
    comb_flag = z(1, dt=torch.int64)
    comb_ptrs = torch.tensor([comb.data_ptr()], dtype=torch.int64, device=dev)
    flag_ptrs = torch.tensor([comb_flag.data_ptr()], dtype=torch.int64, device=dev)
    staging = torch.randn(1, t_cap, k + 1, H, device=dev).to(torch.bfloat16)
    done = z(1, dt=torch.int32)

    def combine_send():
        C.afd_combine_send(staging, rid[0], rwt[0], tcount[0], comb_ptrs, flag_ptrs, done, H,
                           [1, t_cap, k, k + 1, e_local, 0, 1, 0, 1, 1, 0, F, 0, 0])

    out["combine_send_us"] = round(_graph_time_us(combine_send, reps), 2)
    epoch0 = z(1, dt=torch.int64)  # target 0: the wait passes at once

    def combine():
        C.afd_combine(comb, fmask, T, comb_flag, 0, epoch0, F, 10**9)

    out["combine_us"] = round(_graph_time_us(combine, reps), 2)
    torch.cuda.synchronize()
    out["status"] = int(C.read_status(torch.cuda.current_device()))
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--tokens", default="1,43,128,256,1024")
    ap.add_argument("--reps", type=int, default=50)
    args = ap.parse_args(argv)
    for shape in args.shapes.split(","):
        for T in (int(t) for t in args.tokens.split(",")):
            print(json.dumps(run(shape, T, args.reps)), flush=True)


if __name__ == "__main__":
    main()
