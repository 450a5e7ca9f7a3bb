"""CUDA MoE expert path: align -> gather -> tcgen05 grouped GEMMs -> combine.

The two GEMMs run on the 5th-generation tensor cores (``grouped_gemm``, or
``grouped_gemm_w8`` for fp8 block-scaled weights): ``gate_up`` with the
SwiGLU epilogue fused, then ``down``.  No step needs a
host synchronisation, so the whole path captures into a CUDA graph.
"""

from __future__ import annotations

import torch

from afd_plugin_b200.ops._ext import ops as _cuda_ops


def moe_experts_cuda(
    x: torch.Tensor,
    w13: torch.Tensor,
    w2: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    *,
    expert_offset: int = 0,
    w13_scale: torch.Tensor | None = None,
    w2_scale: torch.Tensor | None = None,
    shared_out: torch.Tensor | None = None,
    n_shared: int = 0,
) -> torch.Tensor:
    C = _cuda_ops()
    e_local = w13.shape[0] - n_shared
    ids = topk_ids.to(torch.int32).contiguous()
    counts, offsets, row_token, _row_slot, tsr, total = C.moe_align(ids, e_local, expert_offset, n_shared)
    xs = C.moe_gather(x.contiguous(), row_token, total)
    if w13_scale is not None:
        # fp8 block-scaled experts: the weights stay fp8 in HBM and are
        # dequantised tile by tile in shared memory (W8A16 tcgen05 GEMM).
        ne = w13.shape[0]
        h = C.grouped_gemm_w8(xs, w13, w13_scale, offsets, counts, 1, ne)
        y = C.grouped_gemm_w8(h, w2, w2_scale, offsets, counts, 0, ne)
    else:
        h = C.grouped_gemm(xs, w13, offsets, counts, 1)
        y = C.grouped_gemm(h, w2, offsets, counts, 0)
    return C.moe_combine(y, topk_weights.float().contiguous(), tsr, shared_out)


__all__ = ["moe_experts_cuda"]
