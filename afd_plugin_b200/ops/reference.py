"""Plain PyTorch (fp32-accumulating) definitions of every op the kernels implement.

These are the numerical oracles for the CUDA kernels and the execution path
for CPU runs (unit tests, gloo multi-rank parity).  They are written for
clarity, not speed.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps) * weight.float()).to(x.dtype)


def fused_add_rms_norm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """``residual' = x + residual``; returns ``(rms_norm(residual'), residual')``."""
    new_res = (x.float() + residual.float()).to(residual.dtype)
    return rms_norm(new_res, weight, eps), new_res


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    xf = x.float()
    return (F.silu(xf[..., :d]) * xf[..., d:]).to(x.dtype)


# --------------------------------------------------------------------- RoPE
def rope_cos_sin_cache(
    rotary_dim: int,
    max_positions: int,
    base: float,
    rope_scaling: dict | None = None,
    device: torch.device | str = "cpu",
) -> torch.Tensor:
    """``[max_positions, rotary_dim]`` fp32 table: first half cos, second half sin.

    Supports plain RoPE, linear position interpolation (``type == "linear"``)
    and YaRN (``type == "yarn"``), whose frequency ramp and magnitude
    correction follow the YaRN paper (Peng et al. 2023); other scaling types
    are refused rather than ignored.
    """
    half = rotary_dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim))
    mscale = 1.0
    rs = rope_scaling or {}
    kind = rs.get("type", rs.get("rope_type"))
    if kind in ("yarn", "deepseek_yarn"):
        factor = float(rs["factor"])
        orig = int(rs.get("original_max_position_embeddings", 4096))
        beta_fast = float(rs.get("beta_fast", 32))
        beta_slow = float(rs.get("beta_slow", 1))

        def corr_dim(num_rot: float) -> float:
            return (rotary_dim * math.log(orig / (num_rot * 2 * math.pi))) / (2 * math.log(base))

        low = max(math.floor(corr_dim(beta_fast)), 0)
        high = min(math.ceil(corr_dim(beta_slow)), rotary_dim - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(half, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
        extrap_mask = 1.0 - ramp
        inv_interp = inv_freq / factor
        inv_freq = inv_interp * (1 - extrap_mask) + inv_freq * extrap_mask
        m = float(rs.get("mscale", 1.0))
        m_all = float(rs.get("mscale_all_dim", 0.0) or 0.0)

        def get_m(s: float, mm: float) -> float:
            return 1.0 if s <= 1 else 0.1 * mm * math.log(s) + 1.0

        mscale = get_m(factor, m) / get_m(factor, m_all) if m_all else get_m(factor, m)
    elif kind == "linear":
        inv_freq = inv_freq / float(rs["factor"])  # position interpolation
    elif kind not in (None, "default"):
        raise ValueError(f"unsupported rope_scaling type {kind!r}")
    t = torch.arange(max_positions, dtype=torch.float64)
    freqs = torch.outer(t, inv_freq)
    cache = torch.cat([freqs.cos() * mscale, freqs.sin() * mscale], dim=-1)
    return cache.to(torch.float32).to(device)


def apply_rope(
    x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, *, interleaved: bool
) -> torch.Tensor:
    """Rotate the last dim of ``x`` ``[T, heads, rotary_dim]`` (returns a new tensor).

    ``interleaved`` pairs (0,1),(2,3)... (GPT-J / DeepSeek); otherwise the two
    halves are paired (NeoX / Qwen).
    """
    rot = x.shape[-1]
    half = rot // 2
    cs = cos_sin[positions.long()]
    cos = cs[:, :half].unsqueeze(1)
    sin = cs[:, half:].unsqueeze(1)
    xf = x.float()
    if interleaved:
        x1 = xf[..., 0::2]
        x2 = xf[..., 1::2]
        o1 = x1 * cos - x2 * sin
        o2 = x2 * cos + x1 * sin
        out = torch.stack([o1, o2], dim=-1).flatten(-2)
    else:
        x1 = xf[..., :half]
        x2 = xf[..., half:]
        out = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)
    return out.to(x.dtype)


# ------------------------------------------------------------------ routing
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
    """Return ``(weights fp32 [T,k], ids int32 [T,k])``.

    * sqrtsoftplus scoring (DeepSeek-V4): scores sqrt(softplus(logits)),
      selection like sigmoid scoring.
    * ``forced_ids`` [T, k] (hash routing): experts given, weights gathered
      from the scores.

    * softmax scoring: probabilities over all experts, optional group limit,
      pick top-k probabilities.
    * sigmoid scoring (DeepSeek-V3 ``noaux_tc``): selection uses
      ``sigmoid + bias`` with group scores = sum of each group's top-2, the
      weights are the un-biased sigmoid scores.
    Weights are renormalised to sum 1 when ``renormalize`` and then multiplied
    by ``routed_scaling_factor``.  Ties break toward the lower expert id.
    """
    lf = logits.float()
    T, E = lf.shape
    if scoring == "softmax":
        scores = torch.softmax(lf, dim=-1)
        select = scores
    elif scoring in ("sigmoid", "sqrtsoftplus"):
        scores = torch.sigmoid(lf) if scoring == "sigmoid" else torch.sqrt(torch.nn.functional.softplus(lf))
        select = scores + (bias.float() if bias is not None else 0.0)
    else:
        raise ValueError(f"unknown scoring {scoring!r}")
    if forced_ids is not None:
        # hash routing: the experts are given (per token id); weights from the scores
        ids = forced_ids.long()
        weights = scores.gather(1, ids)
        if renormalize:
            weights = weights / weights.sum(dim=-1, keepdim=True)
        return (weights * routed_scaling_factor).float(), ids.to(torch.int32)
    if n_group > 1 and topk_group < n_group:
        grouped = select.view(T, n_group, E // n_group)
        if scoring == "sigmoid":
            gscore = grouped.topk(2, dim=-1).values.sum(-1)
        else:
            gscore = grouped.max(dim=-1).values
        gidx = _stable_topk(gscore, topk_group)
        gmask = torch.zeros_like(gscore).scatter_(1, gidx, 1.0)
        emask = gmask.unsqueeze(-1).expand(T, n_group, E // n_group).reshape(T, E)
        select = select.masked_fill(emask == 0, float("-inf"))
    ids = _stable_topk(select, top_k)
    weights = scores.gather(1, ids)
    if renormalize:
        weights = weights / weights.sum(dim=-1, keepdim=True)
    weights = weights * routed_scaling_factor
    return weights.float(), ids.to(torch.int32)


def _stable_topk(x: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k indices with ties broken toward the lower index (deterministic)."""
    # A stable ascending sort of -x orders by (-value, index).
    order = torch.argsort(-x.float(), dim=-1, stable=True)
    return order[..., :k]


# ---------------------------------------------------------------------- MoE
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
) -> torch.Tensor:
    """Routed experts: ``sum_k w_k * down(silu(gate(x)) * up(x))``.

    ``w13 [E_local, 2I, H]`` (gate rows then up rows), ``w2 [E_local, H, I]``.
    Ids outside ``[expert_offset, expert_offset + E_local)`` contribute zero
    (expert parallelism).  fp8 weights are dequantised with their block scales.
    """
    T, H = x.shape
    E_local = w13.shape[0]
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    local = topk_ids.long() - expert_offset
    for e in range(E_local):
        tok, slot = torch.nonzero(local == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        a = x[tok].float()
        g_u = dequant_block(w13[e], None if w13_scale is None else w13_scale[e]).float()
        d = dequant_block(w2[e], None if w2_scale is None else w2_scale[e]).float()
        hmid = silu_and_mul(a @ g_u.t())
        y = hmid @ d.t()
        out.index_add_(0, tok, y * topk_weights[tok, slot].float().unsqueeze(-1))
    return out.to(x.dtype)


def dense_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    h = silu_and_mul(x.float() @ w13.float().t())
    return (h @ w2.float().t()).to(x.dtype)


# --------------------------------------------------------------------- fp8
FP8_MAX = 448.0


def quant_fp8_block_weight(w: torch.Tensor, block: tuple[int, int] = (128, 128)) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise ``w [N, K]`` to e4m3 with one fp32 scale per ``block`` tile."""
    N, K = w.shape
    bn, bk = block
    nb, kb = (N + bn - 1) // bn, (K + bk - 1) // bk
    pad = torch.zeros(nb * bn, kb * bk, dtype=torch.float32, device=w.device)
    pad[:N, :K] = w.float()
    tiles = pad.view(nb, bn, kb, bk)
    amax = tiles.abs().amax(dim=(1, 3)).clamp(min=1e-12)
    scale = amax / FP8_MAX
    q = (tiles / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX)
    q = q.view(nb * bn, kb * bk)[:N, :K].to(torch.float8_e4m3fn)
    return q, scale


def dequant_block(w: torch.Tensor, scale: torch.Tensor | None, block: tuple[int, int] = (128, 128)) -> torch.Tensor:
    if scale is None:
        return w
    N, K = w.shape
    bn, bk = block
    s = scale.repeat_interleave(bn, 0)[:N].repeat_interleave(bk, 1)[:, :K]
    return w.float() * s


def quant_fp8_act_1x128(x: torch.Tensor, group: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token, per-128-column e4m3 quantisation: returns ``(q [T,H], scale [T,H/128])``."""
    T, H = x.shape
    g = x.float().view(T, H // group, group)
    amax = g.abs().amax(dim=-1).clamp(min=1e-12)
    scale = amax / FP8_MAX
    q = (g / scale.unsqueeze(-1)).clamp(-FP8_MAX, FP8_MAX).view(T, H).to(torch.float8_e4m3fn)
    return q, scale


def dequant_fp8_act_1x128(q: torch.Tensor, scale: torch.Tensor, group: int = 128) -> torch.Tensor:
    T, H = q.shape
    return (q.float().view(T, H // group, group) * scale.unsqueeze(-1)).view(T, H)


# --------------------------------------------------------------- attention
def gather_paged(cache: torch.Tensor, block_table: torch.Tensor, length: int) -> torch.Tensor:
    """Rows ``0..length-1`` of one sequence from a paged cache ``[nb, bs, ...]``."""
    bs = cache.shape[1]
    nblk = (length + bs - 1) // bs
    rows = cache[block_table[:nblk].long()].flatten(0, 1)
    return rows[:length]


def mla_decode(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
    kv_lora_rank: int,
) -> torch.Tensor:
    """Absorbed MLA decode: ``q [B, H, kv_lora+rope]`` over paged latent KV.

    Returns ``[B, H, kv_lora_rank]`` (latent output before the V up-projection).
    """
    B, Hh, D = q.shape
    out = torch.empty(B, Hh, kv_lora_rank, dtype=q.dtype, device=q.device)
    for b in range(B):
        n = int(seq_lens[b])
        kv = gather_paged(kv_cache, block_table[b], n).float()  # [n, D]
        s = (q[b].float() @ kv.t()) * scale  # [H, n]
        p = torch.softmax(s, dim=-1)
        out[b] = (p @ kv[:, :kv_lora_rank]).to(q.dtype)
    return out


def mla_prefill(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    positions: torch.Tensor,
    scale: float,
    kv_lora_rank: int,
    keep: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal absorbed MLA for ``T`` query tokens of ONE sequence.

    ``keep [T, n]`` (DeepSeek sparse attention) restricts each query to the
    cached positions its indexer selected.
    """
    n = int(positions.max()) + 1
    kv = gather_paged(kv_cache, block_table, n).float()
    s = torch.einsum("thd,nd->thn", q.float(), kv) * scale
    mask = torch.arange(n, device=q.device)[None, :] > positions.long()[:, None]
    if keep is not None:
        mask = mask | ~keep[:, :n]
    s = s.masked_fill(mask[:, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("thn,nd->thd", p, kv[:, :kv_lora_rank]).to(q.dtype)


def dsa_index_scores(q: torch.Tensor, w: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Lightning-indexer scores ``[T, N]``: ``sum_h w[t, h] * relu(q[t, h] . k[n])``.

    ``q [T, heads, d]``, ``w [T, heads]`` (already scaled), ``k [N, d]`` or
    ``[T, N, d]`` (per-query key sets, as in a batched decode step).  The
    DeepSeek-V3.2 indexer (its ``fp8_index``) computes this on fp8 operands;
    here it is fp32.
    """
    if k.dim() == 2:
        logits = torch.einsum("thd,nd->thn", q.float(), k.float())
    else:
        logits = torch.einsum("thd,tnd->thn", q.float(), k.float())
    return torch.einsum("thn,th->tn", logits.clamp_min(0.0), w.float())


def dsa_select(scores: torch.Tensor, valid: torch.Tensor, topk: int) -> torch.Tensor:
    """Positions ``[T, min(topk, N)]`` of the best-scoring valid keys per query; -1 pads.

    Equal scores are common (the ReLU zeroes many of them); ties go to the
    earlier position (a stable sort), so the selection does not depend on how
    many padded columns the score matrix has -- a decode step and a prefill of
    the same tokens select the same positions.
    """
    k = min(int(topk), scores.shape[-1])
    order = scores.masked_fill(~valid, float("-inf")).sort(dim=-1, descending=True, stable=True).indices
    idx = order[..., :k]
    return torch.where(valid.gather(-1, idx), idx, torch.full_like(idx, -1))


def mla_decode_sparse(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    keep_pos: torch.Tensor,
    scale: float,
    kv_lora_rank: int,
) -> torch.Tensor:
    """Absorbed MLA decode over the selected positions ``keep_pos [B, K]`` (-1 = unused) only."""
    bs, D = kv_cache.shape[1], kv_cache.shape[-1]
    pos = keep_pos.long().clamp_min(0)
    slots = block_table.long().gather(1, pos // bs) * bs + pos % bs
    kv = kv_cache.reshape(-1, D)[slots].float()  # [B, K, D]
    s = torch.einsum("bhd,bkd->bhk", q.float(), kv) * scale
    s = s.masked_fill((keep_pos < 0)[:, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhk,bkd->bhd", p, kv[..., :kv_lora_rank]).to(q.dtype)


def gqa_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    """``q [B, Hq, D]`` over paged ``k/v_cache [nb, bs, Hkv, D]``."""
    B, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    g = Hq // Hkv
    out = torch.empty_like(q)
    for b in range(B):
        n = int(seq_lens[b])
        k = gather_paged(k_cache, block_table[b], n).float()  # [n, Hkv, D]
        v = gather_paged(v_cache, block_table[b], n).float()
        qb = q[b].float().view(Hkv, g, D)
        s = torch.einsum("kgd,nkd->kgn", qb, k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("kgn,nkd->kgd", p, v).reshape(Hq, D).to(q.dtype)
    return out


def gqa_prefill(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    positions: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    T, Hq, D = q.shape
    n = int(positions.max()) + 1
    k = gather_paged(k_cache, block_table, n).float()
    v = gather_paged(v_cache, block_table, n).float()
    Hkv = k.shape[1]
    g = Hq // Hkv
    qf = q.float().view(T, Hkv, g, D)
    s = torch.einsum("tkgd,nkd->tkgn", qf, k) * scale
    mask = torch.arange(n, device=q.device)[None, :] > positions.long()[:, None]
    s = s.masked_fill(mask[:, None, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("tkgn,nkd->tkgd", p, v).reshape(T, Hq, D).to(q.dtype)


# ------------------------------------------------------ gated delta net (linear attention)
def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x / sqrt(sum(x^2) + eps) over the last dim, in fp32."""
    xf = x.float()
    return xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, state: torch.Tensor | None = None,
                  activation: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Depthwise causal convolution of one sequence.

    ``x`` [T, C], ``weight`` [C, K]; ``state`` [C, K-1] holds the K-1 inputs
    before x (oldest first), zeros when None.  y[t, c] = sum_j w[c, j] *
    u[t + j, c] over u = [state; x]; SiLU when ``activation``.  Returns
    (y [T, C] fp32, new state [C, K-1] fp32).
    """
    T, C = x.shape
    K = weight.shape[1]
    prev = torch.zeros(C, K - 1, device=x.device) if state is None else state.float()
    u = torch.cat([prev.t(), x.float()], dim=0)  # [K-1+T, C]
    w = weight.float()
    y = torch.zeros(T, C, device=x.device)
    for j in range(K):
        y += u[j : j + T] * w[:, j]
    if activation:
        y = y * torch.sigmoid(y)
    return y, u[T:].t().contiguous()


def gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                     state: torch.Tensor | None = None, scale: float | None = None,
                     qk_l2norm: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Gated delta rule over one sequence, token by token (the recurrent form).

    q, k [T, Hv, dk]; v [T, Hv, dv]; g [T, Hv] log-decay (<= 0); beta [T, Hv];
    state [Hv, dk, dv].  Per token and head, with S the state:
        S = exp(g) S;  S = S + k (beta (v - S^T k))^T;  o = S^T q * scale
    (the gated delta rule of Yang et al., "Gated Delta Networks").  Returns
    (o [T, Hv, dv] fp32, final state fp32).
    """
    T, Hv, dk = q.shape
    dv = v.shape[-1]
    qf, kf = (l2norm(q), l2norm(k)) if qk_l2norm else (q.float(), k.float())
    scale = dk ** -0.5 if scale is None else scale
    S = torch.zeros(Hv, dk, dv, device=q.device) if state is None else state.float().clone()
    out = torch.zeros(T, Hv, dv, device=q.device)
    for t in range(T):
        S = S * torch.exp(g[t].float())[:, None, None]
        kv = torch.einsum("hkv,hk->hv", S, kf[t])
        u = beta[t].float()[:, None] * (v[t].float() - kv)
        S = S + torch.einsum("hk,hv->hkv", kf[t], u)
        out[t] = torch.einsum("hkv,hk->hv", S, qf[t]) * scale
    return out, S


def rms_norm_gated(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dim, times weight, times SiLU(z); fp32 result."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    zf = z.float()
    return y * (zf * torch.sigmoid(zf))


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor,
              dt_bias: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Gated DeltaNet gates: g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b)."""
    g = -torch.exp(A_log.float()) * torch.nn.functional.softplus(a.float() + dt_bias.float())
    return g, torch.sigmoid(b.float())


# ------------------------------------------------------ manifold-constrained hyper-connections
def sinkhorn(logits: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    """Sinkhorn-Knopp projection of exp(logits) [..., n, n] towards a doubly
    stochastic matrix: alternate row and column normalisation ``iters`` times."""
    m = torch.exp(logits.float() - logits.float().amax(dim=(-2, -1), keepdim=True)) + eps
    for _ in range(iters):
        m = m / (m.sum(-1, keepdim=True) + eps)
        m = m / (m.sum(-2, keepdim=True) + eps)
    return m


def mhc_mix(residual: torch.Tensor, fn: torch.Tensor, base: torch.Tensor, scale: torch.Tensor, *, norm_eps: float,
            hc_eps: float, post_alpha: float, sinkhorn_iters: int):
    """Mixing coefficients of one mHC sub-layer from the residual streams.

    residual [T, n, H]; fn [(2 + n) n, n H]; base [(2 + n) n]; scale [3].
    With x = RMSNorm(flatten(residual)) (no weight) and m = x fn^T:
      pre  = sigmoid(scale0 m[:n] + base[:n]) + hc_eps          [T, n]
      post = post_alpha sigmoid(scale1 m[n:2n] + base[n:2n])     [T, n]
      res  = Sinkhorn(scale2 m[2n:] + base[2n:])                 [T, n, n]
    (manifold-constrained hyper-connections, Xie et al., DeepSeek-AI 2025).
    """
    T, n, H = residual.shape
    x = residual.float().reshape(T, n * H)
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + norm_eps)
    m = x @ fn.float().t()
    b = base.float()
    sc = scale.float()
    pre = torch.sigmoid(sc[0] * m[:, :n] + b[:n]) + hc_eps
    post = post_alpha * torch.sigmoid(sc[1] * m[:, n : 2 * n] + b[n : 2 * n])
    res = sinkhorn((sc[2] * m[:, 2 * n :] + b[2 * n :]).view(T, n, n), sinkhorn_iters, hc_eps)
    return pre, post, res


def mhc_pre(residual: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """Sub-layer input: sum_i pre_i * residual_i -> [T, H] fp32."""
    return torch.einsum("tn,tnh->th", pre.float(), residual.float())


def mhc_post(residual: torch.Tensor, out: torch.Tensor, post: torch.Tensor, res: torch.Tensor) -> torch.Tensor:
    """New streams: residual_i' = sum_j res_ij residual_j + post_i * out -> [T, n, H] fp32."""
    return torch.einsum("tij,tjh->tih", res.float(), residual.float()) + post.float()[..., None] * out.float()[:, None]


__all__ = [name for name in globals() if not name.startswith("_") and callable(globals()[name])]
