"""Decoder building blocks with explicit weight tensors.

Each block owns plain tensors (registered as non-trainable parameters) and a
``forward`` made of :mod:`afd_plugin_b200.ops` calls, so the same code runs the
fp32 CPU oracle and the bf16 sm_100a path.
"""

from __future__ import annotations

import math

from dataclasses import dataclass

import torch
from torch import nn

from afd_plugin_b200 import ops
from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.ops import reference as ref


def _param(shape, dtype, device) -> nn.Parameter:
    return nn.Parameter(torch.empty(*shape, dtype=dtype, device=device), requires_grad=False)


@dataclass
class AttentionMetadata:
    """Per-step attention inputs.

    Decode steps: one query token per sequence, ``seq_lens`` includes it.
    Prefill steps: ``prefill_seqs`` lists ``(token_start, token_end, seq_idx)``
    over the flattened token dimension.
    """

    positions: torch.Tensor  # [T] int64
    slot_mapping: torch.Tensor  # [T] int64
    block_table: torch.Tensor  # [B, max_blocks] int32
    seq_lens: torch.Tensor  # [B] int32
    is_decode: bool = True
    prefill_seqs: list[tuple[int, int, int]] | None = None
    # Linear-attention (Gated DeltaNet) layers: per-sequence recurrent state.
    # state_slots [S] picks each sequence's state row, cu_seqlens [S + 1]
    # bounds its tokens, state_reset [S] starts it from a zero state.  None on
    # a decode step means one token per sequence with slot = row.
    state_slots: torch.Tensor | None = None
    cu_seqlens: torch.Tensor | None = None
    state_reset: torch.Tensor | None = None
    # Token ids of the step's rows (hash-routed MoE layers need them).
    input_ids: torch.Tensor | None = None
    # DeepSeek sparse attention, decode steps: some sequence is longer than
    # index_topk, so the indexer must select (a host decision, made before a
    # step so dense steps can replay graphs).
    sparse_decode: bool = False

    def linear_state_args(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
        if self.state_slots is not None:
            return self.cu_seqlens, self.state_slots, self.state_reset
        T = self.num_tokens
        dev = self.positions.device
        rows = torch.arange(T + 1, dtype=torch.int32, device=dev)
        return rows, rows[:T], None

    @property
    def num_tokens(self) -> int:
        return int(self.positions.shape[0])


@dataclass(frozen=True)
class TPInfo:
    """Attention tensor parallelism: this rank's share of the heads.

    Heads are split evenly over ``size`` ranks; the output projection is
    row-parallel, so each rank's partial output is summed over ``group``.
    """

    rank: int = 0
    size: int = 1
    group: object | None = None
    # a peer-memory all-reduce over ``group`` (``parallel/tp_allreduce.py``); NCCL when absent
    peer_ar: object | None = None

    def shard(self, n: int, what: str) -> tuple[int, int]:
        """(first index, count) of this rank's share of ``n`` items."""
        if n % self.size:
            raise ValueError(f"{what}={n} does not split over tensor-parallel size {self.size}")
        per = n // self.size
        return self.rank * per, per

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            if self.peer_ar is not None and x.is_cuda:
                return self.peer_ar(x)
            import torch.distributed as dist

            dist.all_reduce(x, group=self.group)
        return x


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float, dtype, device):
        super().__init__()
        self.eps = eps
        self.weight = _param((dim,), dtype, device)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return ops.rms_norm(x, self.weight, self.eps)
        return ops.fused_add_rms_norm(x, residual, self.weight, self.eps)


class DSAIndexer(nn.Module):
    """Lightning indexer of DeepSeek sparse attention (DeepSeek-V3.2, GLM-MoE-DSA).

    Per token: ``q = wq_b(q_latent)`` split into ``index_n_heads`` heads of
    ``index_head_dim``; ``k = LayerNorm(wk(x))`` (one ``index_head_dim`` row,
    cached per position beside the MLA latent); head weights
    ``weights_proj(x) / sqrt(heads) / sqrt(index_head_dim)``.  The first
    ``qk_rope_head_dim`` dims of q and k are rotated with NeoX pairing.  A
    query scores a cached position ``sum_h w_h * relu(q_h . k)`` and attends
    to the ``index_topk`` best positions at or before it.  This is the indexer
    the reference's DeepSeek-V3.2 path runs on the Attention role
    (``afd_plugin/model_executor/models/deepseek_v2.py:638-650`` allocates its
    top-k buffer there).  DeepSeek rotates q and k by a Hadamard matrix before
    quantising them to fp8; the rotation is orthogonal, so it leaves these
    fp32 scores unchanged and is not applied.
    """

    def __init__(self, arch: ModelArchConfig, dtype, device):
        super().__init__()
        if not arch.q_lora_rank:
            raise ValueError("the DeepSeek sparse-attention indexer reads the q_lora latent")
        H = arch.hidden_size
        self.nh, self.d = arch.index_n_heads, arch.index_head_dim
        self.rope = arch.qk_rope_head_dim
        self.topk = arch.index_topk
        self.wq_b = _param((self.nh * self.d, arch.q_lora_rank), dtype, device)
        self.wk = _param((self.d, H), dtype, device)
        self.k_norm_weight = _param((self.d,), dtype, device)
        self.k_norm_bias = _param((self.d,), dtype, device)
        self.weights_proj = _param((self.nh, H), dtype, device)
        self.w_scale = (self.nh ** -0.5) * (self.d ** -0.5)

    def keys(self, x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
        k = torch.nn.functional.layer_norm(ops.linear(x, self.wk).float(), (self.d,), self.k_norm_weight.float(),
                                           self.k_norm_bias.float(), 1e-6).to(x.dtype)
        ops.rope_(k.view(-1, 1, self.d)[..., : self.rope], positions, cos_sin, interleaved=False)
        return k

    def queries(self, x: torch.Tensor, q_latent: torch.Tensor, positions: torch.Tensor,
                cos_sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        q = ops.linear(q_latent, self.wq_b).view(-1, self.nh, self.d)
        ops.rope_(q[..., : self.rope], positions, cos_sin, interleaved=False)
        return q, ops.linear(x, self.weights_proj).float() * self.w_scale

    def select_decode(self, q: torch.Tensor, w: torch.Tensor, index_cache: torch.Tensor,
                      meta: AttentionMetadata) -> torch.Tensor:
        """Kept positions ``[B, min(topk, max_len)]`` per decode row (-1 pads)."""
        bs = index_cache.shape[1]
        n_max = int(meta.seq_lens.max())
        cols = (n_max + bs - 1) // bs
        B = meta.block_table.shape[0]
        k = index_cache[meta.block_table[:, :cols].long()].view(B, cols * bs, self.d)
        scores = ref.dsa_index_scores(q, w, k)
        valid = torch.arange(cols * bs, device=q.device)[None, :] < meta.seq_lens.long()[:, None]
        return ref.dsa_select(scores, valid, self.topk)

    def select_prefill(self, q: torch.Tensor, w: torch.Tensor, index_cache: torch.Tensor,
                       block_row: torch.Tensor, positions: torch.Tensor) -> torch.Tensor | None:
        """``keep [t, n]`` for one sequence's queries, or None when every query sees all its keys."""
        n = int(positions.max()) + 1
        if n <= self.topk:
            return None
        k = ref.gather_paged(index_cache, block_row, n)
        scores = ref.dsa_index_scores(q, w, k)
        valid = torch.arange(n, device=q.device)[None, :] <= positions.long()[:, None]
        pos = ref.dsa_select(scores, valid, self.topk)
        hits = torch.zeros(pos.shape[0], n, dtype=torch.int32, device=q.device)
        return hits.scatter_add_(1, pos.clamp_min(0), (pos >= 0).int()) > 0


class MLAAttention(nn.Module):
    """DeepSeek multi-head latent attention, absorbed form for cache reads.

    With ``arch.index_topk`` (DeepSeek sparse attention) the layer owns a
    :class:`DSAIndexer` and its cache argument is ``(latent cache, indexer
    key cache)``.  Prefill queries attend to their selected positions; a
    decode step selects only when ``meta.sparse_decode`` (some sequence is
    longer than ``index_topk``), otherwise every position is selected and the
    dense decode kernel runs.
    """

    def __init__(self, arch: ModelArchConfig, dtype, device, tp: TPInfo = TPInfo()):
        super().__init__()
        self.arch = arch
        self.tp = tp
        H = arch.hidden_size
        self.head0, nh = tp.shard(arch.num_attention_heads, "num_attention_heads")
        self.num_heads = nh
        self.qk_nope = arch.qk_nope_head_dim
        self.qk_rope = arch.qk_rope_head_dim
        self.v_dim = arch.v_head_dim
        self.kv_lora = arch.kv_lora_rank
        self.scale = arch.softmax_scale
        qk = arch.qk_head_dim
        # The two projections that read the layer input (q or q_a, and
        # kv_a_proj_with_mqa) share one weight so they run as one GEMM.
        self.n_q_in = arch.q_lora_rank if arch.q_lora_rank else nh * qk
        self.n_in = self.n_q_in + self.kv_lora + self.qk_rope
        self.in_proj = _param((self.n_in, H), dtype, device)
        if arch.q_lora_rank:
            self.q_a_layernorm = RMSNorm(arch.q_lora_rank, arch.rms_norm_eps, dtype, device)
            self.q_b_proj = _param((nh * qk, arch.q_lora_rank), dtype, device)
        self.kv_a_layernorm = RMSNorm(self.kv_lora, arch.rms_norm_eps, dtype, device)
        # Absorbed up-projections derived from kv_b_proj at load time.
        self.w_uk = _param((nh, self.qk_nope, self.kv_lora), dtype, device)
        self.w_uv_t = _param((nh, self.kv_lora, self.v_dim), dtype, device)
        self.o_proj = _param((H, nh * self.v_dim), dtype, device)
        self.indexer = DSAIndexer(arch, dtype, device) if arch.has_indexer else None

    @property
    def q_proj(self) -> torch.Tensor:
        return self.in_proj[: self.n_q_in]

    q_a_proj = q_proj

    @property
    def kv_a_proj_with_mqa(self) -> torch.Tensor:
        return self.in_proj[self.n_q_in : self.n_in]

    def set_kv_b_proj(self, w: torch.Tensor) -> None:
        """Full checkpoint ``kv_b_proj [heads * (nope + v), kv_lora]``; keeps this rank's heads."""
        w = w.view(self.arch.num_attention_heads, self.qk_nope + self.v_dim, self.kv_lora)
        w = w[self.head0 : self.head0 + self.num_heads]
        self.w_uk.data.copy_(w[:, : self.qk_nope, :])
        self.w_uv_t.data.copy_(w[:, self.qk_nope :, :].transpose(1, 2))

    def project(self, h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
        """``(q [T, H, qk], kv_a [T, kv_lora + rope], q_latent [T, q_lora] | None)``; views may be strided."""
        y = ops.linear(h, self.in_proj)
        kv_a = y[:, self.n_q_in : self.n_in]
        q_latent = None
        if self.arch.q_lora_rank:
            q_latent = self.q_a_layernorm(y[:, : self.n_q_in].contiguous())
            q = ops.linear(q_latent, self.q_b_proj)
        else:
            q = y[:, : self.n_q_in]
        return q.view(h.shape[0], self.num_heads, self.qk_nope + self.qk_rope), kv_a, q_latent

    def forward(self, h: torch.Tensor, meta: AttentionMetadata, kv_cache, cos_sin: torch.Tensor):
        index_cache = None
        if isinstance(kv_cache, tuple):
            kv_cache, index_cache = kv_cache
        T = h.shape[0]
        q, kv_a, q_latent = self.project(h)
        q_pe = q[..., self.qk_nope :]
        # latent norm + key rope + cache store, and the query's rope (in place), in one launch
        ops.mla_cache_write(
            kv_cache, kv_a, self.kv_a_layernorm.weight, self.kv_a_layernorm.eps,
            meta.positions, cos_sin, meta.slot_mapping, self.kv_lora, q_pe=q_pe,
        )
        sparse = False
        if self.indexer is not None:
            k_idx = self.indexer.keys(h, meta.positions, cos_sin)
            index_cache.view(-1, self.indexer.d).index_copy_(0, meta.slot_mapping.long(), k_idx)
            sparse = meta.sparse_decode or not meta.is_decode
            if sparse:
                qi, wi = self.indexer.queries(h, q_latent, meta.positions, cos_sin)
        q_nope = q[..., : self.qk_nope]
        if (h.is_cuda and meta.is_decode and not sparse and self.kv_lora == 512 and self.qk_rope == 64
                and self.num_heads % 16 == 0):
            # Head-major end to end: [H,T,128]x[H,128,512] -> kernel -> [H,T,512]x[H,512,v].
            q_lat = torch.bmm(q_nope.transpose(0, 1), self.w_uk)
            o_lat = ops.mla_decode_split(q_lat.transpose(0, 1), q_pe, kv_cache, meta.block_table, meta.seq_lens,
                                         self.scale, head_major_out=True)
            # [H,T,512]x[H,512,v] written straight into token-major rows (ldc = H*v) for o_proj
            o = torch.empty(T, self.num_heads, self.v_dim, dtype=h.dtype, device=h.device)
            torch.bmm(o_lat, self.w_uv_t, out=o.transpose(0, 1))
            return self.tp.all_reduce(ops.linear(o.view(T, self.num_heads * self.v_dim), self.o_proj))
        # [H, T, nope] x [H, nope, kv_lora] -> [H, T, kv_lora]
        if h.is_cuda:
            q_lat = torch.bmm(q_nope.transpose(0, 1), self.w_uk)
        else:
            q_lat = torch.bmm(q_nope.transpose(0, 1).float(), self.w_uk.float()).to(h.dtype)
        q_full = torch.cat([q_lat.transpose(0, 1), q_pe], dim=-1).contiguous()  # [T, H, 576]
        if meta.is_decode and sparse:
            keep_pos = self.indexer.select_decode(qi, wi, index_cache, meta)
            o_lat = ops.mla_decode_sparse(q_full, kv_cache, meta.block_table, meta.seq_lens, keep_pos, self.scale,
                                          self.kv_lora)
        elif meta.is_decode:
            o_lat = ops.mla_decode(q_full, kv_cache, meta.block_table, meta.seq_lens, self.scale, self.kv_lora)
        else:
            o_lat = torch.empty(T, self.num_heads, self.kv_lora, dtype=h.dtype, device=h.device)
            for start, end, seq in meta.prefill_seqs or []:
                keep = None
                if self.indexer is not None:
                    keep = self.indexer.select_prefill(qi[start:end], wi[start:end], index_cache,
                                                       meta.block_table[seq], meta.positions[start:end])
                o_lat[start:end] = ref.mla_prefill(
                    q_full[start:end], kv_cache, meta.block_table[seq], meta.positions[start:end],
                    self.scale, self.kv_lora, keep,
                )
        if h.is_cuda:
            o = torch.bmm(o_lat.transpose(0, 1), self.w_uv_t)  # [H, T, v]
        else:
            o = torch.bmm(o_lat.transpose(0, 1).float(), self.w_uv_t.float()).to(h.dtype)
        o = o.transpose(0, 1).reshape(T, self.num_heads * self.v_dim)
        return self.tp.all_reduce(ops.linear(o, self.o_proj))


class GQAAttention(nn.Module):
    """Grouped-query attention, with per-head QK RMSNorm when ``arch.qk_norm`` (Qwen3);
    without it, the multi-head attention of DeepSeek V1 (``kv heads == heads``)."""

    def __init__(self, arch: ModelArchConfig, dtype, device, tp: TPInfo = TPInfo()):
        super().__init__()
        self.arch = arch
        self.tp = tp
        self.q0, self.nq = tp.shard(arch.num_attention_heads, "num_attention_heads")
        self.kv0, self.nkv = tp.shard(arch.num_key_value_heads, "num_key_value_heads")
        self.d = arch.head_dim
        self.scale = arch.softmax_scale
        H = arch.hidden_size
        self.qkv_proj = _param(((self.nq + 2 * self.nkv) * self.d, H), dtype, device)
        self.qk_norm = arch.qk_norm
        if self.qk_norm:
            self.q_norm = RMSNorm(self.d, arch.rms_norm_eps, dtype, device)
            self.k_norm = RMSNorm(self.d, arch.rms_norm_eps, dtype, device)
        self.o_proj = _param((H, self.nq * self.d), dtype, device)

    def forward(self, h: torch.Tensor, meta: AttentionMetadata, kv_cache: tuple[torch.Tensor, torch.Tensor], cos_sin):
        T = h.shape[0]
        qkv = ops.linear(h, self.qkv_proj)
        k_cache, v_cache = kv_cache
        if h.is_cuda and cos_sin.shape[-1] == self.d and self.d in (32, 64, 128, 256):
            # QK-norm, RoPE and the cache write of k / v in one kernel
            q = ops.gqa_prologue(qkv, self.nq, self.nkv, self.d,
                                 self.q_norm.weight if self.qk_norm else None,
                                 self.k_norm.weight if self.qk_norm else None,
                                 self.q_norm.eps if self.qk_norm else 1e-6,
                                 meta.positions, cos_sin, k_cache, v_cache, meta.slot_mapping)
            return self._attend(q, meta, k_cache, v_cache, T)
        q, k, v = qkv.split([self.nq * self.d, self.nkv * self.d, self.nkv * self.d], dim=-1)
        if self.qk_norm:
            q = self.q_norm(q.reshape(T * self.nq, self.d)).view(T, self.nq, self.d)
            k = self.k_norm(k.reshape(T * self.nkv, self.d)).view(T, self.nkv, self.d)
        else:  # contiguous head rows for the in-place rope and the cache-write kernel
            q = q.reshape(T, self.nq, self.d).contiguous()
            k = k.reshape(T, self.nkv, self.d).contiguous()
        v = v.reshape(T, self.nkv, self.d)
        ops.rope_(q, meta.positions, cos_sin, interleaved=False)
        ops.rope_(k, meta.positions, cos_sin, interleaved=False)
        ops.gqa_cache_write(k_cache, v_cache, k, v, meta.slot_mapping)
        return self._attend(q, meta, k_cache, v_cache, T)

    def _attend(self, q, meta, k_cache, v_cache, T):
        if meta.is_decode:
            o = ops.gqa_decode(q, k_cache, v_cache, meta.block_table, meta.seq_lens, self.scale)
        else:
            from afd_plugin_b200.ops import reference as ref

            o = torch.empty_like(q)
            for start, end, seq in meta.prefill_seqs or []:
                o[start:end] = ref.gqa_prefill(
                    q[start:end], k_cache, v_cache, meta.block_table[seq], meta.positions[start:end], self.scale
                )
        return self.tp.all_reduce(ops.linear(o.reshape(T, self.nq * self.d), self.o_proj))



class GatedDeltaNet(nn.Module):
    """Gated DeltaNet linear attention (Qwen3.5 / Qwen3-Next ``linear_attn``).

    One input projection ``in_proj [conv_dim + value_dim + 2 nv, H]`` with
    rows ordered q | k | v | z | b | a (the checkpoint's per-key-head grouped
    ``in_proj_qkvz`` / ``in_proj_ba`` rows are regrouped at load time), a
    depthwise causal convolution over q | k | v with a rolling state, the gated
    delta rule with an fp32 recurrent state per (sequence, value head), the
    gated RMSNorm and ``out_proj``.  Behaviour of the layer the reference's
    Qwen3.5 wrapper runs natively (``afd_plugin/model_executor/models/qwen3_5.py``,
    Attention-owned ``linear_attn``).
    """

    def __init__(self, arch: ModelArchConfig, dtype, device):
        super().__init__()
        self.arch = arch
        self.nk, self.nv = arch.linear_num_key_heads, arch.linear_num_value_heads
        self.dk, self.dv = arch.linear_key_head_dim, arch.linear_value_head_dim
        self.K = arch.linear_conv_kernel_dim
        self.key_dim, self.value_dim = arch.linear_key_dim, arch.linear_value_dim
        self.conv_dim = arch.linear_conv_dim
        H = arch.hidden_size
        self.in_proj = _param((self.conv_dim + self.value_dim + 2 * self.nv, H), dtype, device)
        self.conv_weight = _param((self.conv_dim, self.K), dtype, device)
        self.A_log = _param((self.nv,), torch.float32, device)
        self.dt_bias = _param((self.nv,), torch.float32, device)
        self.norm_weight = _param((self.dv,), dtype, device)
        self.out_proj = _param((H, self.value_dim), dtype, device)
        self.eps = arch.rms_norm_eps

    # checkpoint layout -> fused rows
    def set_in_proj_qkvz(self, w: torch.Tensor) -> None:
        r = self.nv // self.nk
        g = w.view(self.nk, 2 * self.dk + 2 * r * self.dv, -1)
        q, k = g[:, : self.dk], g[:, self.dk : 2 * self.dk]
        v = g[:, 2 * self.dk : 2 * self.dk + r * self.dv]
        z = g[:, 2 * self.dk + r * self.dv :]
        rows = torch.cat([t.reshape(-1, t.shape[-1]) for t in (q, k, v, z)])
        self.in_proj.data[: self.conv_dim + self.value_dim].copy_(rows.to(self.in_proj.device, self.in_proj.dtype))

    def set_in_proj_ba(self, w: torch.Tensor) -> None:
        r = self.nv // self.nk
        g = w.view(self.nk, 2 * r, -1)
        rows = torch.cat([g[:, :r].reshape(-1, g.shape[-1]), g[:, r:].reshape(-1, g.shape[-1])])
        self.in_proj.data[self.conv_dim + self.value_dim :].copy_(rows.to(self.in_proj.device, self.in_proj.dtype))

    def _cuda_ok(self, h: torch.Tensor) -> bool:
        return (h.is_cuda and self.dk in (32, 64, 128) and self.dv % 32 == 0 and self.dv >= self.dk
                and (self.dk < 128 or self.dv <= 128) and 2 <= self.K <= 8)

    def forward(self, h: torch.Tensor, meta: AttentionMetadata, state: tuple[torch.Tensor, torch.Tensor], cos_sin=None):
        conv_state, ssm_state = state
        proj = ops.linear(h, self.in_proj)
        cd, vd, nv = self.conv_dim, self.value_dim, self.nv
        z = proj[:, cd : cd + vd]
        b = proj[:, cd + vd : cd + vd + nv]
        a = proj[:, cd + vd + nv :]
        cu, slots, reset = meta.linear_state_args()
        if ops.checks.enabled():
            ops.checks.state_slots("gated_delta_net", slots, max_seqs=ssm_state.shape[0])
        if self._cuda_ok(h):
            C = ops._cuda_ops()
            conv = C.gdn_conv(proj[:, :cd], self.conv_weight, conv_state, cu, slots, reset)
            o = C.gdn_recurrent(conv, z, a, b, self.A_log, self.dt_bias, self.norm_weight, self.eps, ssm_state, cu,
                                slots, reset, self.nk)
            return ops.linear(o, self.out_proj)
        return ops.linear(self._forward_reference(proj, z, a, b, conv_state, ssm_state, cu, slots, reset).to(h.dtype),
                          self.out_proj)

    def _forward_reference(self, proj, z, a, b, conv_state, ssm_state, cu, slots, reset) -> torch.Tensor:
        from afd_plugin_b200.ops import reference as ref

        T = proj.shape[0]
        nk, nv, dk, dv = self.nk, self.nv, self.dk, self.dv
        r = nv // nk
        out = torch.empty(T, nv * dv, device=proj.device)
        cu_l = cu.tolist()
        for i, sl in enumerate(slots.tolist()):
            t0, t1 = cu_l[i], cu_l[i + 1]
            fresh = reset is not None and bool(reset[i])
            n = t1 - t0
            if n == 0:
                continue
            conv, new_conv = ref.causal_conv1d(proj[t0:t1, : self.conv_dim], self.conv_weight,
                                               None if fresh else conv_state[sl])
            conv_state[sl].copy_(new_conv.to(conv_state.dtype))
            conv = conv.to(proj.dtype).float()
            q = conv[:, : nk * dk].view(n, nk, dk).repeat_interleave(r, dim=1)
            k = conv[:, nk * dk : 2 * nk * dk].view(n, nk, dk).repeat_interleave(r, dim=1)
            v = conv[:, 2 * nk * dk :].view(n, nv, dv)
            g, beta = ref.gdn_gates(a[t0:t1], b[t0:t1], self.A_log, self.dt_bias)
            o, st = ref.gated_delta_rule(q, k, v, g, beta, None if fresh else ssm_state[sl])
            ssm_state[sl].copy_(st)
            out[t0:t1] = ref.rms_norm_gated(o, z[t0:t1].view(n, nv, dv), self.norm_weight, self.eps).reshape(n, -1)
        return out


class GatedGQAAttention(nn.Module):
    """Full attention of the Qwen3.5 / Qwen3-Next family.

    ``q_proj`` emits a query and an output gate per head (checkpoint rows
    interleaved per head: query d, gate d); per-head QK RMSNorm; RoPE on the
    first ``rotary_dim`` dims (NeoX pairing); GQA over the paged cache;
    ``o_proj(attn * sigmoid(gate))``.
    """

    def __init__(self, arch: ModelArchConfig, dtype, device):
        super().__init__()
        self.arch = arch
        self.nq, self.nkv, self.d = arch.num_attention_heads, arch.num_key_value_heads, arch.head_dim
        self.rot = arch.rotary_dim
        self.scale = 1.0 / math.sqrt(self.d)
        H = arch.hidden_size
        # rows: q (nq d) | gate (nq d) | k (nkv d) | v (nkv d)
        self.qkv_proj = _param(((2 * self.nq + 2 * self.nkv) * self.d, H), dtype, device)
        self.q_norm = RMSNorm(self.d, arch.rms_norm_eps, dtype, device)
        self.k_norm = RMSNorm(self.d, arch.rms_norm_eps, dtype, device)
        self.o_proj = _param((H, self.nq * self.d), dtype, device)

    def set_q_proj(self, w: torch.Tensor) -> None:
        g = w.view(self.nq, 2, self.d, -1)
        nqd = self.nq * self.d
        self.qkv_proj.data[:nqd].copy_(g[:, 0].reshape(nqd, -1).to(self.qkv_proj.device, self.qkv_proj.dtype))
        self.qkv_proj.data[nqd : 2 * nqd].copy_(g[:, 1].reshape(nqd, -1).to(self.qkv_proj.device, self.qkv_proj.dtype))

    def forward(self, h: torch.Tensor, meta: AttentionMetadata, kv_cache: tuple[torch.Tensor, torch.Tensor], cos_sin):
        T = h.shape[0]
        nq, nkv, d = self.nq, self.nkv, self.d
        qkv = ops.linear(h, self.qkv_proj)
        q, gate, k, v = qkv.split([nq * d, nq * d, nkv * d, nkv * d], dim=-1)
        q = self.q_norm(q.reshape(T * nq, d)).view(T, nq, d)
        k = self.k_norm(k.reshape(T * nkv, d)).view(T, nkv, d)
        v = v.reshape(T, nkv, d)
        ops.rope_(q[..., : self.rot], meta.positions, cos_sin, interleaved=False)
        ops.rope_(k[..., : self.rot], meta.positions, cos_sin, interleaved=False)
        k_cache, v_cache = kv_cache
        ops.gqa_cache_write(k_cache, v_cache, k, v, meta.slot_mapping)
        if meta.is_decode:
            o = ops.gqa_decode(q, k_cache, v_cache, meta.block_table, meta.seq_lens, self.scale)
        else:
            from afd_plugin_b200.ops import reference as ref

            o = torch.empty_like(q)
            for start, end, seq in meta.prefill_seqs or []:
                o[start:end] = ref.gqa_prefill(
                    q[start:end], k_cache, v_cache, meta.block_table[seq], meta.positions[start:end], self.scale
                )
        o = o.reshape(T, nq * d) * torch.sigmoid(gate.float()).to(o.dtype)
        return ops.linear(o, self.o_proj)


class DenseMLP(nn.Module):
    """SwiGLU MLP with gate and up stacked in ``w13 [2I, H]``."""

    def __init__(self, hidden: int, inter: int, dtype, device, quant: str | None = None):
        super().__init__()
        wdtype = torch.float8_e4m3fn if quant == "fp8_block" else dtype
        self.quant = quant
        self.w13 = _param((2 * inter, hidden), wdtype, device)
        self.w2 = _param((hidden, inter), wdtype, device)
        if quant == "fp8_block":
            self.w13_scale = _param(((2 * inter + 127) // 128, (hidden + 127) // 128), torch.float32, device)
            self.w2_scale = _param(((hidden + 127) // 128, (inter + 127) // 128), torch.float32, device)
        else:
            self.w13_scale = None
            self.w2_scale = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.quant == "fp8_block":
            if x.is_cuda and x.shape[0] > 0:
                # one-"expert" grouped GEMMs on the fp8 weights (tiles dequantised in shared memory)
                C = ops._cuda_ops()
                T = x.shape[0]
                off = torch.zeros(1, dtype=torch.int32, device=x.device)
                cnt = torch.full((1,), T, dtype=torch.int32, device=x.device)
                h = C.grouped_gemm_w8(x.contiguous(), self.w13.unsqueeze(0), self.w13_scale.unsqueeze(0), off, cnt, 1, 1)
                return C.grouped_gemm_w8(h, self.w2.unsqueeze(0), self.w2_scale.unsqueeze(0), off, cnt, 0, 1)
            from afd_plugin_b200.ops import reference as ref

            w13 = ref.dequant_block(self.w13, self.w13_scale).to(x.dtype)
            w2 = ref.dequant_block(self.w2, self.w2_scale).to(x.dtype)
            return ops.dense_mlp(x, w13, w2)
        return ops.dense_mlp(x, self.w13, self.w2)


class MoEGate(nn.Module):
    """Router.  ``hash_routing`` (DeepSeek-V4 hash layers): the experts come from
    a token-id table ``tid2eid [vocab, k]``; the scores only weight them."""

    def __init__(self, arch: ModelArchConfig, dtype, device, *, hash_routing: bool = False):
        super().__init__()
        self.arch = arch
        self.weight = _param((arch.n_routed_experts, arch.hidden_size), dtype, device)
        self.tid2eid = None
        if hash_routing:
            self.tid2eid = torch.zeros(arch.vocab_size, arch.num_experts_per_tok, dtype=torch.int32, device=device)
            self.e_score_correction_bias = None
        elif arch.topk_method == "noaux_tc":
            self.e_score_correction_bias = _param((arch.n_routed_experts,), torch.float32, device)
        else:
            self.e_score_correction_bias = None

    def finalize(self) -> None:
        """fp32 copy of the gate: router logits are computed in fp32 on every path
        (the fused dispatch kernel accumulates them in fp32 too), so routing
        decisions agree between colocated and disaggregated runs.  A reload
        refreshes the copy in place."""
        w = getattr(self, "weight_f32", None)
        if w is not None and w.shape == self.weight.shape and w.device == self.weight.device:
            w.copy_(self.weight.detach())
        else:
            self.weight_f32 = self.weight.detach().float()

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        if h.is_cuda and h.dtype == self.weight.dtype == torch.bfloat16:
            # bf16 operands, fp32 accumulation and output in one cuBLAS call
            return torch.mm(h, self.weight.t(), out_dtype=torch.float32)
        w = getattr(self, "weight_f32", None)
        if w is None or w.device != h.device:
            w = self.weight.float()
        return h.float() @ w.t()

    def route(self, logits: torch.Tensor, input_ids: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        a = self.arch
        from afd_plugin_b200.models.routing_simulator import balanced_routing_enabled, balanced_topk

        if balanced_routing_enabled():
            return balanced_topk(logits.shape[0], a.n_routed_experts, a.num_experts_per_tok, device=logits.device)
        forced = None
        if self.tid2eid is not None:
            if input_ids is None:
                raise RuntimeError("hash-routed MoE layer needs the tokens' input_ids")
            forced = self.tid2eid[input_ids.long()]
        return ops.topk_route(
            logits,
            a.num_experts_per_tok,
            scoring=a.scoring_func,
            renormalize=a.norm_topk_prob,
            bias=self.e_score_correction_bias,
            n_group=a.n_group if a.topk_method in ("group_limited_greedy", "noaux_tc") else 1,
            topk_group=a.topk_group if a.topk_method in ("group_limited_greedy", "noaux_tc") else 1,
            routed_scaling_factor=a.routed_scaling_factor,
            forced_ids=forced,
        )


class RoutedExperts(nn.Module):
    """Stacked expert weights for the experts ``[offset, offset + n_local)``.

    ``n_extra`` additional slots after the routed experts hold the shared
    experts split into chunks of the routed intermediate size, so the CUDA path
    runs routed and shared experts in one grouped GEMM ("virtual experts").
    """

    def __init__(self, arch: ModelArchConfig, n_local: int, offset: int, dtype, device, n_extra: int = 0):
        super().__init__()
        self.n_local = n_local
        self.n_extra = n_extra
        self.offset = offset
        I, H = arch.moe_intermediate_size, arch.hidden_size
        self.quant = arch.quant
        wdtype = torch.float8_e4m3fn if arch.quant == "fp8_block" else dtype
        self.w13_all = _param((n_local + n_extra, 2 * I, H), wdtype, device)
        self.w2_all = _param((n_local + n_extra, H, I), wdtype, device)
        if arch.quant == "fp8_block":
            self.w13_scale = _param((n_local, (2 * I + 127) // 128, (H + 127) // 128), torch.float32, device)
            self.w2_scale = _param((n_local, (H + 127) // 128, (I + 127) // 128), torch.float32, device)
        else:
            self.w13_scale = None
            self.w2_scale = None

    @property
    def w13(self) -> torch.Tensor:
        return self.w13_all[: self.n_local]

    @property
    def w2(self) -> torch.Tensor:
        return self.w2_all[: self.n_local]

    def pack_shared(self, shared: "DenseMLP") -> None:
        """Copy the shared expert into the extra slots, chunked by the routed width."""
        if not self.n_extra:
            return
        I = self.w2_all.shape[2]
        Is = shared.w2.shape[1]
        for c in range(self.n_extra):
            e = self.n_local + c
            self.w13_all.data[e, :I].copy_(shared.w13[c * I : (c + 1) * I])
            self.w13_all.data[e, I:].copy_(shared.w13[Is + c * I : Is + (c + 1) * I])
            self.w2_all.data[e].copy_(shared.w2[:, c * I : (c + 1) * I])

    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        return ops.moe_experts(
            x, self.w13, self.w2, topk_weights, topk_ids, expert_offset=self.offset,
            w13_scale=self.w13_scale, w2_scale=self.w2_scale,
        )


class MoEBlock(nn.Module):
    """Gate + routed experts (+ shared experts).  ``ep_rank/ep_size`` shard the experts."""

    def __init__(self, arch: ModelArchConfig, dtype, device, *, ep_rank: int = 0, ep_size: int = 1, with_gate: bool = True,
                 layer_idx: int = -1):
        super().__init__()
        self.arch = arch
        E = arch.n_routed_experts
        if E % ep_size:
            raise ValueError(f"{E} experts do not split over {ep_size} expert-parallel ranks")
        n_local = E // ep_size
        self.hash_routing = 0 <= layer_idx < arch.num_hash_layers
        self.gate = MoEGate(arch, dtype, device, hash_routing=self.hash_routing) if with_gate else None
        I, Is = arch.moe_intermediate_size, arch.shared_intermediate_size
        chunked = (Is > 0 and arch.quant is None and I % 64 == 0 and Is % I == 0)
        self.n_shared_chunks = Is // I if chunked else 0
        self.experts = RoutedExperts(arch, n_local, ep_rank * n_local, dtype, device, n_extra=self.n_shared_chunks)
        self.shared_experts = (
            DenseMLP(arch.hidden_size, Is, dtype, device, arch.quant) if arch.has_shared_experts else None
        )
        # Qwen3.5 / Qwen3-Next: the shared expert's output is scaled by sigmoid(x . w) per token.
        self.shared_expert_gate = _param((1, arch.hidden_size), dtype, device) if arch.shared_expert_gate else None

    def finalize(self) -> None:
        if self.shared_experts is not None:
            self.experts.pack_shared(self.shared_experts)
        if self.gate is not None:
            self.gate.finalize()

    def forward(self, h: torch.Tensor, router_logits: torch.Tensor | None = None,
                input_ids: torch.Tensor | None = None) -> torch.Tensor:
        if router_logits is None:
            if self.gate is None:
                raise RuntimeError("MoE block without a gate needs router_logits")
            router_logits = self.gate.logits(h)
        if self.gate is None:
            raise RuntimeError("MoE block needs gate parameters (bias / routing config) to route")
        w, ids = self.gate.route(router_logits, input_ids)
        return self.forward_experts(h, w, ids)

    def forward_experts(self, h: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                        include_shared: bool = True) -> torch.Tensor:
        ex = self.experts
        sg = self.shared_gate(h) if include_shared else None
        if h.is_cuda and include_shared and self.n_shared_chunks:
            # Routed and shared experts in the same grouped GEMMs; with a shared
            # gate its per-token weight rides along as the chunks' routing weight.
            w = topk_weights
            if sg is not None:
                w = torch.cat([topk_weights.float(), sg.expand(-1, self.n_shared_chunks)], dim=1)
            return ops.moe_experts(h, ex.w13_all, ex.w2_all, w, topk_ids, expert_offset=ex.offset,
                                   n_shared=self.n_shared_chunks)
        out = ex(h, topk_weights, topk_ids)
        if include_shared and self.shared_experts is not None:
            s = self.shared_experts(h)
            out = out + (s if sg is None else (s.float() * sg).to(s.dtype))
        return out

    def shared_gate(self, h: torch.Tensor) -> torch.Tensor | None:
        """sigmoid(h . w_sg) [T, 1] fp32, or None without a shared-expert gate."""
        if self.shared_expert_gate is None:
            return None
        return torch.sigmoid(h.float() @ self.shared_expert_gate.float().t())


__all__ = [
    "AttentionMetadata",
    "DenseMLP",
    "GQAAttention",
    "MLAAttention",
    "MoEBlock",
    "MoEGate",
    "RMSNorm",
    "RoutedExperts",
]
