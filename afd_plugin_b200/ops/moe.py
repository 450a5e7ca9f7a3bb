"""CUDA MoE expert path: align -> gather -> tcgen05 grouped GEMMs -> combine.

The two GEMMs run on the 5th-generation tensor cores.  With bf16 weights they
are ONE persistent launch (``moe_ffn``): ``gate_up`` with the SwiGLU epilogue
fused, then ``down``, the down tiles of an expert starting as soon as its
gate_up tiles are stored.  fp8 block-scaled weights use two
``grouped_gemm_w8`` launches.  No step needs a host synchronisation, so the
whole path captures into a CUDA graph.
"""

from __future__ import annotations

import torch

from afd_plugin_b200.ops._ext import ops as _cuda_ops

# Per-device counters of the two-phase expert kernel (zero between launches).
_SYNC: dict[torch.device, torch.Tensor] = {}
_SYNC_LEN = 4096


def moe_sync_buffer(device: torch.device, experts: int) -> torch.Tensor:
    """The counters a ``moe_ffn`` launch over ``experts`` segments uses on ``device``.

    Allocated once per device (first use comes from an eager step, before any
    graph capture) and shared by every launch on that device's stream.
    """
    if experts + 1 > _SYNC_LEN:
        raise ValueError(f"moe_ffn supports at most {_SYNC_LEN - 1} expert segments per launch, got {experts}")
    device = torch.device(device)
    buf = _SYNC.get(device)
    if buf is None:
        buf = torch.zeros(_SYNC_LEN, dtype=torch.int32, device=device)
        _SYNC[device] = buf
    return buf


_WS: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}
_WS_FLOATS = 4 << 20  # 16 MiB of fp32 partial sums


def gemm_workspace(device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-K workspace of the dense tcgen05 GEMM on ``device``: fp32 partial sums and
    per-tile arrival counters, both zero between launches (every launch leaves them zero).
    Allocated once per device on first use (an eager step, before any graph capture)."""
    device = torch.device(device)
    ws = _WS.get(device)
    if ws is None:
        ws = (torch.zeros(_WS_FLOATS, dtype=torch.float32, device=device),
              torch.zeros(4096, dtype=torch.int32, device=device))
        _WS[device] = ws
    return ws


def moe_rows_hint(tokens: int, top_k: int, experts: int, n_shared: int = 0, shared_rows: int | None = None) -> int:
    """Largest expert segment a decode step expects: twice the mean routed load, or a shared chunk's rows."""
    routed = 2 * (tokens * top_k + experts - 1) // max(1, experts)
    shared = (tokens if shared_rows is None else shared_rows) if n_shared else 0
    # a few whole-batch segments among many small ones: 128-token passes keep the pipeline deep
    return max(1, routed, min(shared, 128))


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
        y = C.moe_ffn(xs, w13, w2, offsets, counts, moe_sync_buffer(x.device, w13.shape[0]),
                      moe_rows_hint(x.shape[0], topk_ids.shape[1], e_local, n_shared))
    return C.moe_combine(y, topk_weights.float().contiguous(), tsr, shared_out)


__all__ = ["gemm_workspace", "moe_experts_cuda", "moe_rows_hint", "moe_sync_buffer"]
