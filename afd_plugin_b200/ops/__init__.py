"""Operator entry points used by the models and the runtime.

Every function takes the same arguments on CPU and CUDA.  CPU tensors run the
plain PyTorch definitions in :mod:`afd_plugin_b200.ops.reference` (the numeric
oracle and the path of the gloo multi-rank tests); CUDA tensors run the
sm_100a kernels of the in-tree extension, which must be built -- a missing
library raises rather than falling back.
"""

from __future__ import annotations

import os

import torch

from afd_plugin_b200.ops import checks
from afd_plugin_b200.ops import reference as ref
from afd_plugin_b200.ops._ext import ops as _cuda_ops

SCORING_IDS = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


def _rows16(t: torch.Tensor) -> bool:
    """Every row of ``t`` (last dim contiguous) starts on a 16-byte boundary and holds whole 16-byte vectors."""
    vec = 16 // t.element_size()
    return (t.stride(-1) == 1 and t.shape[-1] % vec == 0 and t.data_ptr() % 16 == 0
            and all(st % vec == 0 for st in t.stride()[:-1]))


# ----------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if _cuda(x):
        return _cuda_ops().rms_norm(x, weight, eps)
    return ref.rms_norm(x, weight, eps)


def fused_add_rms_norm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(rms_norm(x + residual), x + residual)``; CUDA updates ``residual`` in place."""
    if _cuda(x):
        y = _cuda_ops().fused_add_rms_norm(x, residual, weight, eps)
        return y, residual
    return ref.fused_add_rms_norm(x, residual, weight, eps)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    if _cuda(x):
        return _cuda_ops().silu_and_mul(x)
    return ref.silu_and_mul(x)


# ------------------------------------------------------------------ RoPE
def rope_(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, *, interleaved: bool) -> torch.Tensor:
    """Rotate ``x [T, heads, rot]`` in place (last dim contiguous); returns ``x``."""
    if _cuda(x):
        _cuda_ops().rope_(x, positions, cos_sin, interleaved)
        return x
    x.copy_(ref.apply_rope(x, positions, cos_sin, interleaved=interleaved))
    return x


# --------------------------------------------------------------- routing
def topk_route(
    logits: torch.Tensor,
    top_k: int,
    *,
    scoring: str = "softmax",
    renormalize: bool = False,
    bias: torch.Tensor | None = None,
    n_group: int = 1,
    topk_group: int = 1,
    routed_scaling_factor: float = 1.0,
    forced_ids: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    if forced_ids is not None and checks.enabled():
        checks.expert_ids("topk_route", forced_ids, num_experts=logits.shape[-1])
    if _cuda(logits):
        forced = None if forced_ids is None else forced_ids.to(torch.int32).contiguous()
        return _cuda_ops().topk_route(
            logits, top_k, SCORING_IDS[scoring], renormalize, bias, n_group, topk_group, routed_scaling_factor, forced
        )
    return ref.topk_route(
        logits,
        top_k,
        scoring=scoring,
        renormalize=renormalize,
        bias=bias,
        n_group=n_group,
        topk_group=topk_group,
        routed_scaling_factor=routed_scaling_factor,
        forced_ids=forced_ids,
    )


# -------------------------------------------------------------- attention
def mla_decode(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
    kv_lora_rank: int,
    *,
    num_splits: int = 0,
) -> torch.Tensor:
    if checks.enabled():
        checks.paged_attention("mla_decode", block_table, seq_lens, num_blocks=kv_cache.shape[0],
                               block_size=kv_cache.shape[1])
    if _cuda(q):
        if q.shape[-1] == 576 and kv_lora_rank == 512 and q.shape[1] % 16 == 0:
            return _cuda_ops().mla_decode(q[..., :512], q[..., 512:], kv_cache, block_table, seq_lens, scale,
                                          num_splits, False)
        # The kernel is specialised to DeepSeek's 512 + 64 latent; other
        # (test-sized) shapes run the batched PyTorch form.
        return _mla_decode_torch(q, kv_cache, block_table, seq_lens, scale, kv_lora_rank)
    return ref.mla_decode(q, kv_cache, block_table, seq_lens, scale, kv_lora_rank)


def _mla_decode_torch(q, kv_cache, block_table, seq_lens, scale, kv_lora_rank):
    B, Hh, D = q.shape
    bs = kv_cache.shape[1]
    nblk = block_table.shape[1]
    kv = kv_cache[block_table.long()].view(B, nblk * bs, D).float()
    s = torch.einsum("bhd,bnd->bhn", q.float(), kv) * scale
    mask = torch.arange(nblk * bs, device=q.device)[None, :] >= seq_lens.long()[:, None]
    s = s.masked_fill(mask[:, None, :], float("-inf"))
    return torch.einsum("bhn,bnd->bhd", torch.softmax(s, dim=-1), kv[..., :kv_lora_rank]).to(q.dtype)


def mla_decode_split(
    q_lat: torch.Tensor,
    q_pe: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
    *,
    head_major_out: bool = True,
    num_splits: int = 0,
) -> torch.Tensor:
    """MLA decode with the query as two strided views ``[B, H, 512]`` / ``[B, H, 64]``.

    Returns ``[H, B, 512]`` (head-major, ready for the per-head V up-projection)
    or ``[B, H, 512]``.  CUDA only (the kernel's native interface).
    """
    if checks.enabled():
        checks.paged_attention("mla_decode", block_table, seq_lens, num_blocks=kv_cache.shape[0],
                               block_size=kv_cache.shape[1])
    return _cuda_ops().mla_decode(q_lat, q_pe, kv_cache, block_table, seq_lens, scale, num_splits, head_major_out)


def mla_decode_sparse(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    keep_pos: torch.Tensor,
    scale: float,
    kv_lora_rank: int,
    *,
    num_splits: int = 0,
) -> torch.Tensor:
    """MLA decode over the positions a DeepSeek-sparse-attention indexer kept.

    ``keep_pos [B, K]`` lists each row's selected positions (-1 = unused).
    On a GPU (DeepSeek's 512 + 64 latent, heads a multiple of 16) the sm_100a
    sparse decode kernel gathers the kept rows (``csrc/mla_decode.cu``,
    ``kSparse``) when the layer has at most 32 heads; with more heads its
    16-head CTAs each gather the rows again and the gather plus two batched
    GEMMs is faster (measured on B200: 16 heads 789 vs 1,983 us, 128 heads
    1,248 vs 1,141 us; ``bench/mla_decode_bench.py --sparse``).
    ``AFD_SPARSE_MLA_KERNEL=1`` / ``0`` forces one or the other.
    """
    if checks.enabled():
        checks.paged_attention("mla_decode_sparse", block_table, seq_lens, num_blocks=kv_cache.shape[0],
                               block_size=kv_cache.shape[1])
        bad = (keep_pos >= seq_lens.view(-1, 1).to(keep_pos.dtype)).any()
        if bool(bad):
            raise checks.KernelInputError("mla_decode_sparse: a kept position lies beyond its sequence")
    if (_cuda(q) and sparse_kernel_enabled(q.shape[1]) and q.dtype == torch.bfloat16 and q.shape[-1] == 576
            and kv_lora_rank == 512 and q.shape[1] % 16 == 0):
        return _cuda_ops().mla_decode_sparse(q, kv_cache, block_table, seq_lens.to(torch.int32),
                                             keep_pos.to(torch.int32).contiguous(), scale, num_splits)
    return ref.mla_decode_sparse(q, kv_cache, block_table, keep_pos, scale, kv_lora_rank)


def sparse_kernel_enabled(heads: int = 16) -> bool:
    """Whether sparse MLA decode runs on the gather kernel for ``heads`` heads
    (default: up to 32 heads; ``AFD_SPARSE_MLA_KERNEL=1`` / ``0`` forces it)."""
    v = os.environ.get("AFD_SPARSE_MLA_KERNEL", "")
    if v in ("1", "true", "on"):
        return True
    if v in ("0", "false", "off"):
        return False
    return heads <= 32


def gqa_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
    *,
    num_splits: int = 0,
) -> torch.Tensor:
    if checks.enabled():
        checks.paged_attention("gqa_decode", block_table, seq_lens, num_blocks=k_cache.shape[0],
                               block_size=k_cache.shape[1])
    if _cuda(q):
        if q.shape[-1] == 128 and q.shape[1] // k_cache.shape[2] <= 16 and k_cache.shape[1] % 32 == 0:
            return _cuda_ops().gqa_decode(q.contiguous(), k_cache, v_cache, block_table, seq_lens, scale, num_splits)
        return _gqa_decode_torch(q, k_cache, v_cache, block_table, seq_lens, scale)
    return ref.gqa_decode(q, k_cache, v_cache, block_table, seq_lens, scale)


def _gqa_decode_torch(q, k_cache, v_cache, block_table, seq_lens, scale):
    """Batched GQA decode in PyTorch ops (paged gather + masked softmax)."""
    B, Hq, D = q.shape
    bs, Hkv = k_cache.shape[1], k_cache.shape[2]
    nblk = block_table.shape[1]
    k = k_cache[block_table.long()].view(B, nblk * bs, Hkv, D)
    v = v_cache[block_table.long()].view(B, nblk * bs, Hkv, D)
    g = Hq // Hkv
    s = torch.einsum("bkgd,bnkd->bkgn", q.view(B, Hkv, g, D).float(), k.float()) * scale
    mask = torch.arange(nblk * bs, device=q.device)[None, :] >= seq_lens.long()[:, None]
    s = s.masked_fill(mask[:, None, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bkgn,bnkd->bkgd", p, v.float()).reshape(B, Hq, D).to(q.dtype)


def mla_cache_write(
    kv_cache: torch.Tensor,
    kv_a: torch.Tensor,
    norm_weight: torch.Tensor,
    eps: float,
    positions: torch.Tensor,
    cos_sin: torch.Tensor,
    slot_mapping: torch.Tensor,
    kv_lora_rank: int,
    q_pe: torch.Tensor | None = None,
) -> None:
    """Normalise the latent, rotate the shared rope key and store both in the cache.

    ``kv_a [T, kv_lora + rope]`` is the ``kv_a_proj_with_mqa`` output.  With
    ``q_pe [T, H, rope]`` the query's rope part is rotated in place as well
    (interleaved pairs, like the key), in the same CUDA launch.
    """
    if checks.enabled():
        checks.cache_slots("mla_cache_write", slot_mapping, num_slots=kv_cache.shape[0] * kv_cache.shape[1])
    if _cuda(kv_a):
        if q_pe is not None and not _rows16(q_pe):
            rope_(q_pe, positions, cos_sin, interleaved=True)  # unaligned rows: the separate rope kernel
            q_pe = None
        _cuda_ops().mla_cache_write(kv_cache, kv_a, norm_weight, eps, positions, cos_sin, slot_mapping, kv_lora_rank,
                                    q_pe)
        return
    if q_pe is not None:
        rope_(q_pe, positions, cos_sin, interleaved=True)
    latent = ref.rms_norm(kv_a[:, :kv_lora_rank], norm_weight, eps)
    k_pe = ref.apply_rope(kv_a[:, None, kv_lora_rank:], positions, cos_sin, interleaved=True)[:, 0]
    flat = kv_cache.view(-1, kv_cache.shape[-1])
    flat[slot_mapping.long()] = torch.cat([latent, k_pe], dim=-1).to(kv_cache.dtype)


def gqa_cache_write(
    k_cache: torch.Tensor, v_cache: torch.Tensor, k: torch.Tensor, v: torch.Tensor, slot_mapping: torch.Tensor
) -> None:
    if checks.enabled():
        checks.cache_slots("gqa_cache_write", slot_mapping, num_slots=k_cache.shape[0] * k_cache.shape[1])
    if _cuda(k):
        _cuda_ops().gqa_cache_write(k_cache, v_cache, k, v, slot_mapping)
        return
    kf = k_cache.view(-1, *k_cache.shape[2:])
    vf = v_cache.view(-1, *v_cache.shape[2:])
    kf[slot_mapping.long()] = k.to(k_cache.dtype)
    vf[slot_mapping.long()] = v.to(v_cache.dtype)


def gqa_prologue(
    qkv: torch.Tensor,
    nq: int,
    nkv: int,
    head_dim: int,
    q_norm_w: torch.Tensor | None,
    k_norm_w: torch.Tensor | None,
    eps: float,
    positions: torch.Tensor,
    cos_sin: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> torch.Tensor:
    """GQA attention prologue: optional per-head q / k RMSNorm, NeoX RoPE on
    whole heads, k / v into the paged caches; returns q ``[T, nq, head_dim]``.

    ``qkv [T, (nq + 2 nkv) * head_dim]`` is the fused projection's output.  On
    a GPU one kernel does all of it (one CTA per token); on CPU the same steps
    run one by one.
    """
    if checks.enabled():
        checks.cache_slots("gqa_prologue", slot_mapping, num_slots=k_cache.shape[0] * k_cache.shape[1])
    if _cuda(qkv):
        return _cuda_ops().gqa_prologue(qkv, nq, nkv, head_dim, q_norm_w, k_norm_w, eps, positions, cos_sin, k_cache,
                                        v_cache, slot_mapping)
    T = qkv.shape[0]
    q, k, v = qkv.split([nq * head_dim, nkv * head_dim, nkv * head_dim], dim=-1)
    q = q.reshape(T, nq, head_dim)
    k = k.reshape(T, nkv, head_dim)
    if q_norm_w is not None:
        q = ref.rms_norm(q, q_norm_w, eps).to(qkv.dtype)
    if k_norm_w is not None:
        k = ref.rms_norm(k, k_norm_w, eps).to(qkv.dtype)
    q = ref.apply_rope(q, positions, cos_sin, interleaved=False).to(qkv.dtype)
    k = ref.apply_rope(k, positions, cos_sin, interleaved=False).to(qkv.dtype)
    gqa_cache_write(k_cache, v_cache, k, v.reshape(T, nkv, head_dim), slot_mapping)
    return q


# -------------------------------------------------------------------- MoE
def moe_experts(
    x: torch.Tensor,
    w13: torch.Tensor,
    w2: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    *,
    expert_offset: int = 0,
    w13_scale: torch.Tensor | None = None,
    w2_scale: torch.Tensor | None = None,
    n_shared: int = 0,
) -> torch.Tensor:
    """Routed-expert output ``[T, H]`` (weights applied, summed over k).

    With ``n_shared`` the last ``n_shared`` experts of ``w13``/``w2`` are shared
    chunks applied to every token with weight 1 (CUDA path).
    """
    if checks.enabled():
        checks.expert_ids("moe_experts", topk_ids, weights=topk_weights)
    if _cuda(x):
        from afd_plugin_b200.ops.moe import moe_experts_cuda

        return moe_experts_cuda(
            x, w13, w2, topk_weights, topk_ids, expert_offset=expert_offset, w13_scale=w13_scale, w2_scale=w2_scale,
            n_shared=n_shared,
        )
    if n_shared:
        raise ValueError("virtual shared experts are a CUDA-path layout")
    return ref.moe_experts(
        x, w13, w2, topk_weights, topk_ids, expert_offset=expert_offset, w13_scale=w13_scale, w2_scale=w2_scale
    )


def _tc_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Shapes the tcgen05 GEMM takes: bf16, N % 128 == 0, K % 64 == 0, 16-byte aligned rows."""
    return (x.dtype == w.dtype == torch.bfloat16 and w.dim() == 2 and w.is_contiguous()
            and w.shape[0] % 128 == 0 and w.shape[1] % 64 == 0 and x.dim() == 2 and x.stride(1) == 1
            and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0)


def dense_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """SwiGLU MLP (a dense layer).  CUDA: cuBLAS GEMMs plus the SiLU-mul kernel
    (``dense_ffn``, the one-launch tcgen05 version, is slower at 256-token
    decode batches: its down projection has only H / 128 weight tiles)."""
    if _cuda(x):
        return torch.mm(silu_and_mul(torch.mm(x, w13.t())), w2.t())
    return ref.dense_mlp(x, w13, w2)


def linear(x: torch.Tensor, w: torch.Tensor, *, n_valid: int = 0, out_f32: bool = False) -> torch.Tensor:
    """``x @ w.T`` (cuBLAS on CUDA, fp32-accumulating reference on CPU).

    ``n_valid`` keeps the first ``n_valid`` output columns (a weight padded with
    zero rows); ``out_f32`` returns fp32 logits.  The dense decode projections
    stay on cuBLAS: the tcgen05 kernel here streams weights with the tokens as
    the MMA's N operand, which wins for expert segments of a few dozen tokens
    (``moe_ffn``) but loses 4-5x to cuBLAS's token-tiled kernels at 256-token
    dense projections (``tc_gemm``, measured in ``bench/grouped_gemm_bench.py
    --dense``).
    """
    if _cuda(x):
        y = torch.mm(x, w.t(), out_dtype=torch.float32) if out_f32 else torch.mm(x, w.t())
        return y[:, :n_valid] if n_valid else y
    y = x.float() @ w.float().t()
    y = y if out_f32 else y.to(x.dtype)
    return y[:, :n_valid] if n_valid else y


def head_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Per-head product ``x [E, T, K]`` x ``w [E, N, K]`` -> ``[T, E * N]`` token-major (cuBLAS on CUDA)."""
    E, T, _ = x.shape
    if x.is_cuda:
        y = torch.bmm(x, w.transpose(1, 2))
    else:
        y = torch.bmm(x.float(), w.float().transpose(1, 2)).to(x.dtype)
    return y.transpose(0, 1).reshape(T, E * w.shape[1])


def argmax(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token per row (int32), lowest index on ties; reads bf16 logits in place on CUDA."""
    if _cuda(logits) and logits.dim() == 2 and logits.stride(1) == 1:
        return _cuda_ops().argmax_rows(logits)
    return torch.argmax(logits.float(), dim=-1).to(torch.int32)


__all__ = [
    "argmax",
    "dense_mlp",
    "fused_add_rms_norm",
    "gqa_cache_write",
    "gqa_decode",
    "head_linear",
    "linear",
    "mla_cache_write",
    "mla_decode",
    "moe_experts",
    "rms_norm",
    "rope_",
    "silu_and_mul",
    "topk_route",
]
