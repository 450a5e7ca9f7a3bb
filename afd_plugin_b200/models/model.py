"""Role-aware causal LM shared by the DeepSeek and Qwen3-MoE wrappers.

A model instance is built for one of three roles:

* ``colocated`` -- every module (single-process serving, parity oracle);
* ``attention`` -- embeddings, attention, norms, LM head (plus the MoE gate
  and dense MLPs when ``compute_gate_on_attention``);
* ``ffn`` -- dense MLPs and MoE blocks; experts are sharded over the FFN ranks
  (expert parallelism, ``ep_rank``/``ep_size``).

Behaviour follows the reference wrappers
(``afd_plugin/model_executor/models/deepseek_v2.py:292-599`` and
``qwen3_moe.py:102-321``): the Attention side hands post-attention-norm hidden
states to the FFN side per layer; with ``compute_gate_on_attention`` the MoE
gate runs on the Attention side and dense layers stay local.

Weights are described by :class:`ParamSpec` entries named like the
HuggingFace checkpoint, which drives both safetensors loading and the seeded
random initialisation (per-name seeds, so split roles and the colocated model
hold bit-identical weights).
"""

from __future__ import annotations

import zlib
from collections.abc import Callable, Iterator
from dataclasses import dataclass

import torch
from torch import nn

from afd_plugin_b200 import ops
from afd_plugin_b200.connectors.metadata import AFDExpertRoutingSpec
from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.models.layers import (
    AttentionMetadata,
    DenseMLP,
    GatedDeltaNet,
    GatedGQAAttention,
    GQAAttention,
    MLAAttention,
    MoEBlock,
    RMSNorm,
    TPInfo,
    _param,
)
from afd_plugin_b200.ops import reference as ref

ROLES = ("colocated", "attention", "ffn")
_ATTN = frozenset({"attention"})
_FFN = frozenset({"ffn"})
_BOTH = frozenset({"attention", "ffn"})


@dataclass
class ParamSpec:
    name: str  # HF checkpoint name
    shape: tuple[int, ...]
    setter: Callable[[torch.Tensor], None]
    init: str = "normal"  # "normal" | "ones" | "zeros"
    # fp8-quantised target: random init quantises, checkpoints may carry a scale.
    fp8_scale_name: str | None = None
    # init == "custom": the random-init value comes from make()
    make: Callable[[], torch.Tensor] | None = None


def weight_roles(name: str, arch: ModelArchConfig, *, compute_gate_on_attention: bool,
                 route_on_attention: bool = False) -> frozenset[str]:
    """Which AFD role(s) need checkpoint tensor ``name``.

    Same classification as ``_checkpoint_weight_roles`` of the reference
    (``deepseek_v2.py:69-92``, ``qwen3_moe.py:51-62``).
    """
    parts = name.split(".")
    if arch.hc_mult:
        return _v4_weight_roles(name, parts, route_on_attention=route_on_attention)
    for i, p in enumerate(parts[:-2]):
        if p != "layers":
            continue
        try:
            layer = int(parts[i + 1])
        except ValueError:
            continue
        stage = parts[i + 2]
        rest = parts[i + 3 :]
        if stage in ("self_attn", "linear_attn"):
            return _ATTN
        if stage != "mlp":
            return _BOTH
        if not arch.is_moe_layer(layer):
            return _ATTN if compute_gate_on_attention else _FFN
        if rest and rest[0] == "gate" and (compute_gate_on_attention or route_on_attention):
            return _BOTH
        return _FFN
    return _BOTH


def _v4_weight_roles(name: str, parts: list[str], *, route_on_attention: bool) -> frozenset[str]:
    """DeepSeek-V4 naming (reference ``deepseek_v4.py:45-60``): the ``ffn`` stage of a
    layer is FFN-owned, every other layer stage and the ``hc_head`` tensors are
    Attention-owned, other top-level tensors are needed by both."""
    if parts[-1].startswith("hc_head"):
        return _ATTN
    for i, p in enumerate(parts[:-2]):
        if p != "layers":
            continue
        try:
            int(parts[i + 1])
        except ValueError:
            continue
        stage = parts[i + 2]
        if stage == "ffn":
            if route_on_attention and len(parts) > i + 3 and parts[i + 3] == "gate":
                return _BOTH
            return _FFN
        return _ATTN
    return _BOTH


class DecoderLayer(nn.Module):
    def __init__(self, arch: ModelArchConfig, idx: int, role: str, dtype, device, *, gate_on_attn: bool,
                 ep_rank: int, ep_size: int, route_on_attn: bool = False, tp: TPInfo = TPInfo()):
        super().__init__()
        self.idx = idx
        self.is_moe = arch.is_moe_layer(idx)
        eps = arch.rms_norm_eps
        has_attn = role in ("colocated", "attention")
        self.input_layernorm = RMSNorm(arch.hidden_size, eps, dtype, device) if has_attn else None
        self.post_attention_layernorm = RMSNorm(arch.hidden_size, eps, dtype, device) if has_attn else None
        self.self_attn = None
        self.is_linear_attn = arch.is_linear_attention_layer(idx)
        if has_attn:
            if (self.is_linear_attn or arch.attn_output_gate) and tp.size > 1:
                raise NotImplementedError("attention tensor parallelism covers MLA and GQA attention")
            if self.is_linear_attn:
                self.self_attn = GatedDeltaNet(arch, dtype, device)
            elif arch.attn_output_gate:
                self.self_attn = GatedGQAAttention(arch, dtype, device)
            elif arch.is_mla:
                self.self_attn = MLAAttention(arch, dtype, device, tp)
            else:
                self.self_attn = GQAAttention(arch, dtype, device, tp)
        self.mlp: nn.Module | None = None
        self.gate_only = None
        if role == "colocated":
            self.mlp = MoEBlock(arch, dtype, device, layer_idx=idx) if self.is_moe else DenseMLP(
                arch.hidden_size, arch.intermediate_size, dtype, device, arch.quant)
        elif role == "attention":
            if self.is_moe and (gate_on_attn or route_on_attn):
                from afd_plugin_b200.models.layers import MoEGate

                self.gate_only = MoEGate(arch, dtype, device, hash_routing=idx < arch.num_hash_layers)
            elif gate_on_attn:
                self.mlp = DenseMLP(arch.hidden_size, arch.intermediate_size, dtype, device, arch.quant)
        else:  # ffn
            if self.is_moe:
                self.mlp = MoEBlock(arch, dtype, device, ep_rank=ep_rank, ep_size=ep_size, layer_idx=idx)
            elif not gate_on_attn:
                self.mlp = DenseMLP(arch.hidden_size, arch.intermediate_size, dtype, device, arch.quant)


class AFDCausalLM(nn.Module):
    """Decoder-only MoE LM split by AFD role."""

    family = "base"

    def __init__(
        self,
        arch: ModelArchConfig,
        *,
        role: str = "colocated",
        dtype: torch.dtype = torch.bfloat16,
        device: torch.device | str = "cpu",
        compute_gate_on_attention: bool = False,
        ep_rank: int = 0,
        ep_size: int = 1,
        max_positions: int | None = None,
        route_on_attention: bool = False,
        tp: TPInfo = TPInfo(),
    ):
        super().__init__()
        if role not in ROLES:
            raise ValueError(f"role must be one of {ROLES}, got {role!r}")
        self._validate_arch(arch)
        self.arch = arch
        self.role = role
        self.dtype = dtype
        self.device = torch.device(device)
        self.compute_gate_on_attention = compute_gate_on_attention
        # Routing on the Attention side without moving dense MLPs there (fused connector).
        self.route_on_attention = route_on_attention
        self.ep_rank, self.ep_size = ep_rank, ep_size
        self.tp = tp
        has_attn = role in ("colocated", "attention")
        self.embed_tokens = _param((arch.vocab_size, arch.hidden_size), dtype, device) if has_attn else None
        self.layers = nn.ModuleList(
            DecoderLayer(arch, i, role, dtype, device, gate_on_attn=compute_gate_on_attention,
                         ep_rank=ep_rank, ep_size=ep_size, route_on_attn=route_on_attention, tp=tp)
            for i in range(arch.num_hidden_layers)
        )
        self.norm = RMSNorm(arch.hidden_size, arch.rms_norm_eps, dtype, device) if has_attn else None
        if has_attn and arch.tie_word_embeddings:
            self.lm_head = self.embed_tokens  # tied: the checkpoint carries no lm_head.weight
        else:
            self.lm_head = _param((arch.vocab_size, arch.hidden_size), dtype, device) if has_attn else None
        self.cos_sin = None
        if has_attn:
            rot = arch.rotary_dim
            npos = max_positions or min(arch.max_position_embeddings, 8192)
            self.cos_sin = ref.rope_cos_sin_cache(rot, npos, arch.rope_theta, arch.rope_scaling, device)

    # ----------------------------------------------------------- checks
    def _validate_arch(self, arch: ModelArchConfig) -> None:
        pass

    # ----------------------------------------------------------- forward
    @property
    def num_layers(self) -> int:
        return self.arch.num_hidden_layers

    @property
    def cache_arch(self) -> ModelArchConfig:
        """Shapes of this rank's KV cache (a tensor-parallel GQA rank caches its own KV heads)."""
        if self.tp.size > 1 and not self.arch.is_mla:
            return self.arch.scaled(num_key_value_heads=self.arch.num_key_value_heads // self.tp.size)
        return self.arch

    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.embed_tokens[input_ids.long()]

    def run_attention(self, layer_idx: int, h: torch.Tensor, residual: torch.Tensor | None,
                      meta: AttentionMetadata, kv_cache) -> tuple[torch.Tensor, torch.Tensor]:
        layer = self.layers[layer_idx]
        if residual is None:
            residual = h.clone()
            x = layer.input_layernorm(h)
        else:
            x, residual = layer.input_layernorm(h, residual)
        return layer.self_attn(x, meta, kv_cache, self.cos_sin), residual

    def post_attention_norm(self, layer_idx: int, attn_out: torch.Tensor, residual: torch.Tensor):
        return self.layers[layer_idx].post_attention_layernorm(attn_out, residual)

    def compute_router_logits(self, layer_idx: int, h: torch.Tensor) -> torch.Tensor:
        layer = self.layers[layer_idx]
        gate = layer.gate_only if layer.gate_only is not None else layer.mlp.gate
        return gate.logits(h)

    def compute_ffn_output(self, hidden_states: torch.Tensor, layer_idx: int, **kwargs) -> torch.Tensor:
        layer = self.layers[layer_idx]
        if layer.mlp is None:
            raise RuntimeError(f"layer {layer_idx} FFN is not owned by role {self.role!r}")
        if self.role == "ffn" and self.compute_gate_on_attention and layer.is_moe:
            raise RuntimeError("Attention-side gate: the FFN role must call compute_experts_output")
        if layer.is_moe and kwargs.get("input_ids") is not None:
            return layer.mlp(hidden_states, input_ids=kwargs["input_ids"])
        return layer.mlp(hidden_states)

    def ffn_extra(self, layer_idx: int, residual) -> dict:
        """Extra tensors the FFN of ``layer_idx`` needs besides the hidden states."""
        return {}

    def ffn_needs_input_ids(self, layer_idx: int) -> bool:
        return False

    # Whether the post-attention step is residual add + RMSNorm (the fused
    # dispatch kernel runs it); models with other residual schemes return False.
    fused_post_norm = True

    def compute_experts_output(self, hidden_states: torch.Tensor, layer_idx: int,
                               router_logits: torch.Tensor) -> torch.Tensor:
        layer = self.layers[layer_idx]
        if not (self.compute_gate_on_attention and layer.is_moe):
            raise RuntimeError("compute_experts_output requires an Attention-side-gate MoE layer")
        return layer.mlp(hidden_states, router_logits=router_logits)

    def final_logits(self, h: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        x, _ = self.norm(h, residual)
        return ops.linear(x, self.lm_head)

    def get_experts_layer_indices(self) -> tuple[int, ...]:
        return self.arch.moe_layer_indices

    def get_experts_routing_spec(self, layer_idx: int) -> AFDExpertRoutingSpec:
        return AFDExpertRoutingSpec(router_logits_width=self.arch.n_routed_experts,
                                    router_logits_dtype=torch.float32)

    def ffn_layer_indices(self) -> tuple[int, ...]:
        """Layers whose FFN runs on the FFN role."""
        if self.compute_gate_on_attention:
            return self.arch.moe_layer_indices
        return tuple(range(self.num_layers))

    # ----------------------------------------------------------- weights
    def param_specs(self) -> Iterator[ParamSpec]:
        a = self.arch
        if self.embed_tokens is not None:
            yield ParamSpec("model.embed_tokens.weight", tuple(self.embed_tokens.shape), _copy(self.embed_tokens))
            yield ParamSpec("model.norm.weight", (a.hidden_size,), _copy(self.norm.weight), "ones")
            if not a.tie_word_embeddings:
                yield ParamSpec("lm_head.weight", tuple(self.lm_head.shape), _copy(self.lm_head))
        for i, layer in enumerate(self.layers):
            p = f"model.layers.{i}."
            if layer.input_layernorm is not None:
                yield ParamSpec(p + "input_layernorm.weight", (a.hidden_size,), _copy(layer.input_layernorm.weight), "ones")
                yield ParamSpec(p + "post_attention_layernorm.weight", (a.hidden_size,),
                                _copy(layer.post_attention_layernorm.weight), "ones")
                yield from self._attn_specs(p + "self_attn.", layer.self_attn)
            if layer.gate_only is not None:
                yield from _gate_specs(p + "mlp.gate.", layer.gate_only)
            mlp = layer.mlp
            if isinstance(mlp, DenseMLP):
                yield from _mlp_specs(p + "mlp.", mlp, a.intermediate_size)
            elif isinstance(mlp, MoEBlock):
                if mlp.gate is not None:
                    yield from _gate_specs(p + "mlp.gate.", mlp.gate)
                ex = mlp.experts
                I = a.moe_intermediate_size
                for le in range(ex.n_local):
                    e = ex.offset + le
                    q = f"{p}mlp.experts.{e}."
                    s13 = None if ex.w13_scale is None else ex.w13_scale[le]
                    s2 = None if ex.w2_scale is None else ex.w2_scale[le]
                    yield from _swiglu_specs(q, ex.w13[le], ex.w2[le], s13, s2, I, a.hidden_size)
                if mlp.shared_experts is not None:
                    yield from _mlp_specs(p + "mlp.shared_experts.", mlp.shared_experts, a.shared_intermediate_size)

    def _attn_specs(self, p: str, attn) -> Iterator[ParamSpec]:
        raise NotImplementedError

    def reload_weights(self, checkpoint: str | None = None, *, seed: int = 0) -> None:
        """Reload every parameter of this role in place.

        ``checkpoint`` is an HF safetensors directory; without one the seeded
        random init runs again.  Parameters keep their storage, so CUDA graphs
        captured against them, the fused connector's cached weight views and
        peer-visible pointers stay valid.  Counterpart of the FFN runner's
        ``reload_weights`` (``afd_plugin/v1/worker/ffn_model_runner.py:288-291``),
        which rebuilds the model instead.
        """
        ptrs = {id(p): p.data_ptr() for p in self.parameters()}
        if checkpoint is None:
            self.init_random(seed)
        else:
            from afd_plugin_b200.models.loader import load_checkpoint

            load_checkpoint(self, checkpoint)
        self.finalize_weights()
        moved = [p for p in self.parameters() if ptrs.get(id(p)) != p.data_ptr()]
        if moved:
            raise RuntimeError(f"reload_weights reallocated {len(moved)} parameters")

    def finalize_weights(self) -> None:
        """Derived layouts after loading (shared experts packed as virtual experts)."""
        for layer in self.layers:
            if isinstance(layer.mlp, MoEBlock):
                layer.mlp.finalize()
            if layer.gate_only is not None:
                layer.gate_only.finalize()

    def init_random(self, seed: int = 0, std: float = 0.02, *, generate_on: str | None = None) -> None:
        """Seeded N(0, std) init; each tensor's stream depends only on (seed, name).

        Values are drawn on the model's device unless ``generate_on="cpu"``
        (CPU and CUDA generators produce different streams; generate on CPU to
        compare a GPU model with a CPU one).
        """
        for spec in self.param_specs():
            gen_dev = torch.device(generate_on) if generate_on else (
                self.device if self.device.type == "cuda" else torch.device("cpu"))
            g = torch.Generator(device=gen_dev)
            g.manual_seed((seed * 1_000_003 + zlib.crc32(spec.name.encode())) & 0x7FFFFFFFFFFFFFFF)
            if spec.init == "custom" and spec.make is not None:
                t = spec.make()
            elif spec.init == "ones":
                t = torch.ones(spec.shape, dtype=torch.float32, device=gen_dev)
            elif spec.init == "zeros":
                t = torch.zeros(spec.shape, dtype=torch.float32, device=gen_dev)
            else:
                t = torch.empty(spec.shape, dtype=torch.float32, device=gen_dev).normal_(0.0, std, generator=g)
            spec.setter(t)


def _copy(dst: torch.Tensor) -> Callable[[torch.Tensor], None]:
    def setter(src: torch.Tensor) -> None:
        if tuple(src.shape) != tuple(dst.shape):
            raise ValueError(f"shape mismatch {tuple(src.shape)} vs {tuple(dst.shape)}")
        dst.data.copy_(src.to(dst.device, dst.dtype))

    return setter


def _rows(dst: torch.Tensor, start: int, stop: int) -> Callable[[torch.Tensor], None]:
    def setter(src: torch.Tensor) -> None:
        dst.data[start:stop].copy_(src.to(dst.device, dst.dtype))

    return setter


def _rows_of(dst: torch.Tensor, dst0: int, src0: int, n: int) -> Callable[[torch.Tensor], None]:
    """Copy rows [src0, src0 + n) of a full checkpoint tensor into dst rows [dst0, dst0 + n)."""

    def setter(src: torch.Tensor) -> None:
        dst.data[dst0 : dst0 + n].copy_(src[src0 : src0 + n].to(dst.device, dst.dtype))

    return setter


def _cols_of(dst: torch.Tensor, src0: int) -> Callable[[torch.Tensor], None]:
    """Copy columns [src0, src0 + dst.shape[1]) of a full checkpoint tensor into dst."""

    def setter(src: torch.Tensor) -> None:
        dst.data.copy_(src[:, src0 : src0 + dst.shape[1]].to(dst.device, dst.dtype))

    return setter


def _fp8_rows(dst_w: torch.Tensor, dst_s: torch.Tensor, start: int, stop: int) -> Callable[[torch.Tensor], None]:
    """Setter for an fp8 block-quantised slice: quantises unless given e4m3 data."""

    def setter(src: torch.Tensor) -> None:
        if src.dtype == torch.float8_e4m3fn:
            dst_w.data[start:stop].copy_(src.to(dst_w.device))
            return
        q, s = ref.quant_fp8_block_weight(src.float())
        dst_w.data[start:stop].copy_(q.to(dst_w.device))
        dst_s.data[start // 128 : (stop + 127) // 128].copy_(s.to(dst_s.device))

    return setter


def _swiglu_specs(p: str, w13: torch.Tensor, w2: torch.Tensor, s13, s2, inter: int, hidden: int) -> Iterator[ParamSpec]:
    if s13 is None:
        yield ParamSpec(p + "gate_proj.weight", (inter, hidden), _rows(w13, 0, inter))
        yield ParamSpec(p + "up_proj.weight", (inter, hidden), _rows(w13, inter, 2 * inter))
        yield ParamSpec(p + "down_proj.weight", (hidden, inter), _copy(w2))
        return
    if inter % 128:
        raise ValueError("fp8 block quantisation needs the intermediate size to be a multiple of 128")
    yield ParamSpec(p + "gate_proj.weight", (inter, hidden), _fp8_rows(w13, s13, 0, inter),
                    fp8_scale_name=p + "gate_proj.weight_scale_inv")
    yield ParamSpec(p + "up_proj.weight", (inter, hidden), _fp8_rows(w13, s13, inter, 2 * inter),
                    fp8_scale_name=p + "up_proj.weight_scale_inv")
    yield ParamSpec(p + "down_proj.weight", (hidden, inter), _fp8_rows(w2, s2, 0, hidden),
                    fp8_scale_name=p + "down_proj.weight_scale_inv")


def _mlp_specs(p: str, mlp: DenseMLP, inter: int) -> Iterator[ParamSpec]:
    hidden = mlp.w13.shape[1]
    yield from _swiglu_specs(p, mlp.w13, mlp.w2, mlp.w13_scale, mlp.w2_scale, inter, hidden)


def _gqa_specs(p: str, attn: GQAAttention, a: ModelArchConfig) -> Iterator[ParamSpec]:
    """Full checkpoint shapes of ``q/k/v/o_proj`` (+ QK norms); a tensor-parallel rank keeps its heads."""
    d, nq, nkv = attn.d, attn.nq, attn.nkv
    H, nq_all, nkv_all = a.hidden_size, a.num_attention_heads, a.num_key_value_heads
    yield ParamSpec(p + "q_proj.weight", (nq_all * d, H), _rows_of(attn.qkv_proj, 0, attn.q0 * d, nq * d))
    yield ParamSpec(p + "k_proj.weight", (nkv_all * d, H), _rows_of(attn.qkv_proj, nq * d, attn.kv0 * d, nkv * d))
    yield ParamSpec(p + "v_proj.weight", (nkv_all * d, H),
                    _rows_of(attn.qkv_proj, (nq + nkv) * d, attn.kv0 * d, nkv * d))
    if attn.qk_norm:
        yield ParamSpec(p + "q_norm.weight", (d,), _copy(attn.q_norm.weight), "ones")
        yield ParamSpec(p + "k_norm.weight", (d,), _copy(attn.k_norm.weight), "ones")
    yield ParamSpec(p + "o_proj.weight", (H, nq_all * d), _cols_of(attn.o_proj, attn.q0 * d))


def _gate_specs(p: str, gate) -> Iterator[ParamSpec]:
    yield ParamSpec(p + "weight", tuple(gate.weight.shape), _copy(gate.weight))
    if gate.e_score_correction_bias is not None:
        yield ParamSpec(p + "e_score_correction_bias", tuple(gate.e_score_correction_bias.shape),
                        _copy(gate.e_score_correction_bias), "zeros")


class AFDDeepseekV2ForCausalLM(AFDCausalLM):
    """DeepSeek-V2/V3 family (MLA + DeepSeek MoE)."""

    family = "deepseek"

    def _validate_arch(self, arch: ModelArchConfig) -> None:
        if not arch.is_mla:
            raise ValueError("DeepSeek wrapper requires MLA attention")

    def _attn_specs(self, p: str, attn: MLAAttention) -> Iterator[ParamSpec]:
        """Full checkpoint shapes; a tensor-parallel rank keeps its heads' rows / columns."""
        a = self.arch
        H, nh_all = a.hidden_size, a.num_attention_heads
        qk = a.qk_head_dim
        nq = attn.n_q_in
        nkv = a.kv_lora_rank + a.qk_rope_head_dim
        h0, nh = attn.head0, attn.num_heads
        if a.q_lora_rank:
            yield ParamSpec(p + "q_a_proj.weight", (nq, H), _rows(attn.in_proj, 0, nq))
            yield ParamSpec(p + "q_a_layernorm.weight", (a.q_lora_rank,), _copy(attn.q_a_layernorm.weight), "ones")
            yield ParamSpec(p + "q_b_proj.weight", (nh_all * qk, a.q_lora_rank), _rows_of(attn.q_b_proj, 0, h0 * qk, nh * qk))
        else:
            yield ParamSpec(p + "q_proj.weight", (nh_all * qk, H), _rows_of(attn.in_proj, 0, h0 * qk, nh * qk))
        yield ParamSpec(p + "kv_a_proj_with_mqa.weight", (nkv, H), _rows(attn.in_proj, nq, nq + nkv))
        yield ParamSpec(p + "kv_a_layernorm.weight", (a.kv_lora_rank,), _copy(attn.kv_a_layernorm.weight), "ones")
        shape = (nh_all * (a.qk_nope_head_dim + a.v_head_dim), a.kv_lora_rank)
        yield ParamSpec(p + "kv_b_proj.weight", shape, lambda t, _a=attn: _a.set_kv_b_proj(t.to(_a.w_uk.device, _a.w_uk.dtype)))
        yield ParamSpec(p + "o_proj.weight", (H, nh_all * a.v_head_dim), _cols_of(attn.o_proj, h0 * a.v_head_dim))
        ix = attn.indexer
        if ix is not None:  # replicated on every tensor-parallel rank
            q = p + "indexer."
            yield ParamSpec(q + "wq_b.weight", tuple(ix.wq_b.shape), _copy(ix.wq_b))
            yield ParamSpec(q + "wk.weight", tuple(ix.wk.shape), _copy(ix.wk))
            yield ParamSpec(q + "k_norm.weight", tuple(ix.k_norm_weight.shape), _copy(ix.k_norm_weight), "ones")
            yield ParamSpec(q + "k_norm.bias", tuple(ix.k_norm_bias.shape), _copy(ix.k_norm_bias), "zeros")
            yield ParamSpec(q + "weights_proj.weight", tuple(ix.weights_proj.shape), _copy(ix.weights_proj))


class AFDDeepseekV3ForCausalLM(AFDDeepseekV2ForCausalLM):
    pass


class AFDDeepseekForCausalLM(AFDDeepseekV2ForCausalLM):
    """DeepSeek V1 (DeepSeekMoE): multi-head attention (``q/k/v/o_proj``, no QK
    norm) with the DeepSeek MoE; MLA checkpoints of this class name load as V2.
    The reference picks the same split by ``model_type == "deepseek"``
    (``afd_plugin/model_executor/models/deepseek_v2.py:333-337``)."""

    def _validate_arch(self, arch: ModelArchConfig) -> None:
        if not arch.is_mla and arch.qk_norm:
            raise ValueError("DeepSeek V1 attention has no QK norm")

    def _attn_specs(self, p: str, attn) -> Iterator[ParamSpec]:
        if self.arch.is_mla:
            yield from super()._attn_specs(p, attn)
        else:
            yield from _gqa_specs(p, attn, self.arch)


class AFDGlmMoeDsaForCausalLM(AFDDeepseekV2ForCausalLM):
    pass


class AFDQwen3MoeForCausalLM(AFDCausalLM):
    """Qwen3-MoE (GQA + QK-norm, routed experts only, gate on the FFN side)."""

    family = "qwen3_moe"

    def __init__(self, arch: ModelArchConfig, **kw):
        if kw.get("compute_gate_on_attention"):
            raise ValueError("Qwen3-MoE AFD supports compute_gate_on_attention=false only")
        super().__init__(arch, **kw)

    def _validate_arch(self, arch: ModelArchConfig) -> None:
        if arch.is_mla or not arch.qk_norm:
            raise ValueError("Qwen3-MoE wrapper requires GQA attention with QK-norm")

    def _attn_specs(self, p: str, attn: GQAAttention) -> Iterator[ParamSpec]:
        yield from _gqa_specs(p, attn, self.arch)


class AFDDeepseekV4ForCausalLM(AFDDeepseekV2ForCausalLM):
    """DeepSeek-V4 family: MLA attention, manifold-constrained hyper-connections
    (mHC: ``hc_mult`` residual streams mixed per sub-layer), hash-routed MoE in
    the first ``num_hash_layers`` layers, sqrt-softplus routing scores.

    The AFD split sits around each layer's FFN, as in the reference wrapper
    (``afd_plugin/model_executor/models/deepseek_v4.py:122-283``): the
    Attention side keeps every mHC stream and mixing parameter and sends the
    normalised FFN input plus the token ids (hash routing); the FFN side runs
    the MoE.  The residual travelling between hooks is the tuple
    ``(streams [T, n, H] fp32, post [T, n], res [T, n, n], input_ids)``.
    """

    family = "deepseek_v4"
    fused_post_norm = False
    post_alpha = 2.0

    def __init__(self, arch: ModelArchConfig, **kw):
        super().__init__(arch, **kw)
        n, H = arch.hc_mult, arch.hidden_size
        mix = (2 + n) * n
        dev = self.device
        if self.role in ("colocated", "attention"):
            for layer in self.layers:
                layer.hc_attn_fn = _param((mix, n * H), torch.float32, dev)
                layer.hc_attn_base = _param((mix,), torch.float32, dev)
                layer.hc_attn_scale = _param((3,), torch.float32, dev)
                layer.hc_ffn_fn = _param((mix, n * H), torch.float32, dev)
                layer.hc_ffn_base = _param((mix,), torch.float32, dev)
                layer.hc_ffn_scale = _param((3,), torch.float32, dev)
            self.hc_head_fn = _param((n, n * H), torch.float32, dev)
            self.hc_head_base = _param((n,), torch.float32, dev)
            self.hc_head_scale = _param((1,), torch.float32, dev)

    def _validate_arch(self, arch: ModelArchConfig) -> None:
        if not arch.is_mla or arch.hc_mult < 1:
            raise ValueError("DeepSeek-V4 wrapper requires MLA attention and hc_mult >= 1")

    # ------------------------------------------------------------- mHC
    def _mix(self, fn, base, scale, streams):
        a = self.arch
        return ref.mhc_mix(streams, fn, base, scale, norm_eps=a.rms_norm_eps, hc_eps=a.hc_eps,
                           post_alpha=self.post_alpha, sinkhorn_iters=a.hc_sinkhorn_iters)

    def run_attention(self, layer_idx, h, residual, meta, kv_cache):
        layer = self.layers[layer_idx]
        if residual is None:  # embeddings: every stream starts as the token embedding
            ids = meta.input_ids
            streams = h.float()[:, None, :].expand(h.shape[0], self.arch.hc_mult, h.shape[1]).contiguous()
        else:
            streams, post, res, ids = residual
            streams = ref.mhc_post(streams, h, post, res)
        pre, post, res = self._mix(layer.hc_attn_fn, layer.hc_attn_base, layer.hc_attn_scale, streams)
        x = layer.input_layernorm(ref.mhc_pre(streams, pre).to(self.dtype))
        return layer.self_attn(x, meta, kv_cache, self.cos_sin), (streams, post, res, ids)

    def post_attention_norm(self, layer_idx, attn_out, residual):
        layer = self.layers[layer_idx]
        streams, post, res, ids = residual
        streams = ref.mhc_post(streams, attn_out, post, res)
        pre, post, res = self._mix(layer.hc_ffn_fn, layer.hc_ffn_base, layer.hc_ffn_scale, streams)
        x = layer.post_attention_layernorm(ref.mhc_pre(streams, pre).to(self.dtype))
        return x, (streams, post, res, ids)

    def final_logits(self, h, residual):
        a = self.arch
        streams, post, res, _ = residual
        streams = ref.mhc_post(streams, h, post, res)
        T = streams.shape[0]
        xf = streams.reshape(T, -1)
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + a.rms_norm_eps)
        w = torch.sigmoid(self.hc_head_scale[0] * (xf @ self.hc_head_fn.t()) + self.hc_head_base) + a.hc_eps
        x = self.norm(torch.einsum("tn,tnh->th", w, streams).to(self.dtype))
        return ops.linear(x, self.lm_head)

    def ffn_extra(self, layer_idx, residual) -> dict:
        if self.ffn_needs_input_ids(layer_idx):
            return {"input_ids": residual[3]}
        return {}

    def ffn_needs_input_ids(self, layer_idx: int) -> bool:
        return self.arch.is_moe_layer(layer_idx) and layer_idx < self.arch.num_hash_layers

    # ----------------------------------------------------------- weights
    def param_specs(self) -> Iterator[ParamSpec]:
        a = self.arch
        H = a.hidden_size
        if self.embed_tokens is not None:
            yield ParamSpec("model.embed_tokens.weight", tuple(self.embed_tokens.shape), _copy(self.embed_tokens))
            yield ParamSpec("model.norm.weight", (H,), _copy(self.norm.weight), "ones")
            if not a.tie_word_embeddings:
                yield ParamSpec("lm_head.weight", tuple(self.lm_head.shape), _copy(self.lm_head))
            yield ParamSpec("model.hc_head_fn", tuple(self.hc_head_fn.shape), _copy(self.hc_head_fn))
            yield ParamSpec("model.hc_head_base", tuple(self.hc_head_base.shape), _copy(self.hc_head_base), "zeros")
            yield ParamSpec("model.hc_head_scale", (1,), _copy(self.hc_head_scale), "ones")
        for i, layer in enumerate(self.layers):
            p = f"model.layers.{i}."
            if layer.input_layernorm is not None:
                yield ParamSpec(p + "attn_norm.weight", (H,), _copy(layer.input_layernorm.weight), "ones")
                yield ParamSpec(p + "ffn_norm.weight", (H,), _copy(layer.post_attention_layernorm.weight), "ones")
                for which in ("attn", "ffn"):
                    fn, base, sc = (getattr(layer, f"hc_{which}_{x}") for x in ("fn", "base", "scale"))
                    yield ParamSpec(p + f"hc_{which}_fn", tuple(fn.shape), _copy(fn))
                    yield ParamSpec(p + f"hc_{which}_base", tuple(base.shape), _copy(base), "zeros")
                    yield ParamSpec(p + f"hc_{which}_scale", (3,), _copy(sc), "ones")
                yield from self._attn_specs(p + "attn.", layer.self_attn)
            if layer.gate_only is not None:
                yield from _v4_gate_specs(p + "ffn.gate.", layer.gate_only, a)
            mlp = layer.mlp
            if isinstance(mlp, DenseMLP):
                yield from _mlp_specs(p + "ffn.", mlp, a.intermediate_size)
            elif isinstance(mlp, MoEBlock):
                if mlp.gate is not None:
                    yield from _v4_gate_specs(p + "ffn.gate.", mlp.gate, a)
                ex = mlp.experts
                for le in range(ex.n_local):
                    q = f"{p}ffn.experts.{ex.offset + le}."
                    s13 = None if ex.w13_scale is None else ex.w13_scale[le]
                    s2 = None if ex.w2_scale is None else ex.w2_scale[le]
                    yield from _swiglu_specs(q, ex.w13[le], ex.w2[le], s13, s2, a.moe_intermediate_size, H)
                if mlp.shared_experts is not None:
                    yield from _mlp_specs(p + "ffn.shared_experts.", mlp.shared_experts, a.shared_intermediate_size)


def _v4_gate_specs(p: str, gate, arch: ModelArchConfig) -> Iterator[ParamSpec]:
    yield ParamSpec(p + "weight", tuple(gate.weight.shape), _copy(gate.weight))
    if gate.e_score_correction_bias is not None:
        yield ParamSpec(p + "e_score_correction_bias", tuple(gate.e_score_correction_bias.shape),
                        _copy(gate.e_score_correction_bias), "zeros")
    if gate.tid2eid is not None:
        V, k, E = arch.vocab_size, arch.num_experts_per_tok, arch.n_routed_experts

        def table() -> torch.Tensor:  # seeded stand-in: k distinct experts per token id
            v = torch.arange(V)[:, None]
            return ((v * 7919 + torch.arange(k)[None, :] * (E // k + 1)) % E).to(torch.float32)

        yield ParamSpec(p + "tid2eid", (V, k), lambda t, _g=gate: _g.tid2eid.copy_(t.to(torch.int32)), "custom",
                        make=table)


def _copy_plus_one(dst: torch.Tensor) -> Callable[[torch.Tensor], None]:
    """Zero-centred RMSNorm weight: the checkpoint stores (w - 1)."""

    def setter(src: torch.Tensor) -> None:
        dst.data.copy_((src.float() + 1.0).to(dst.device, dst.dtype))

    return setter


class AFDQwen3_5MoeForCausalLM(AFDCausalLM):
    """Qwen3.5 / Qwen3-Next MoE: Gated DeltaNet + gated full attention, MoE with a gated shared expert.

    Roles as in the reference wrapper (``afd_plugin/model_executor/models/qwen3_5.py:46-73``):
    ``linear_attn`` / ``self_attn`` / norms / embeddings / LM head on the
    Attention side; the MoE gate, routed experts, shared expert and shared-expert
    gate on the FFN side (the gate is also loaded on the Attention side when the
    fused connector routes there).  Text-only.
    """

    family = "qwen3_5"

    def _validate_arch(self, arch: ModelArchConfig) -> None:
        if arch.layer_types is None or not arch.attn_output_gate or arch.is_mla:
            raise ValueError("Qwen3.5 wrapper requires hybrid layer_types with gated GQA full attention")
        if arch.first_k_dense_replace or arch.moe_layer_freq != 1:
            raise ValueError("Qwen3.5 wrapper expects every layer to be an MoE layer")

    def param_specs(self) -> Iterator[ParamSpec]:
        a = self.arch
        H = a.hidden_size
        if self.embed_tokens is not None:
            yield ParamSpec("model.embed_tokens.weight", tuple(self.embed_tokens.shape), _copy(self.embed_tokens))
            yield ParamSpec("model.norm.weight", (H,), _copy_plus_one(self.norm.weight), "zeros")
            if not a.tie_word_embeddings:
                yield ParamSpec("lm_head.weight", tuple(self.lm_head.shape), _copy(self.lm_head))
        for i, layer in enumerate(self.layers):
            p = f"model.layers.{i}."
            if layer.input_layernorm is not None:
                yield ParamSpec(p + "input_layernorm.weight", (H,), _copy_plus_one(layer.input_layernorm.weight), "zeros")
                yield ParamSpec(p + "post_attention_layernorm.weight", (H,),
                                _copy_plus_one(layer.post_attention_layernorm.weight), "zeros")
                if layer.is_linear_attn:
                    yield from self._linear_attn_specs(p + "linear_attn.", layer.self_attn)
                else:
                    yield from self._gated_attn_specs(p + "self_attn.", layer.self_attn)
            if layer.gate_only is not None:
                yield from _gate_specs(p + "mlp.gate.", layer.gate_only)
            mlp = layer.mlp
            if isinstance(mlp, MoEBlock):
                if mlp.gate is not None:
                    yield from _gate_specs(p + "mlp.gate.", mlp.gate)
                ex = mlp.experts
                I = a.moe_intermediate_size
                for le in range(ex.n_local):
                    q = f"{p}mlp.experts.{ex.offset + le}."
                    yield from _swiglu_specs(q, ex.w13[le], ex.w2[le], None, None, I, H)
                if mlp.shared_experts is not None:
                    yield from _mlp_specs(p + "mlp.shared_expert.", mlp.shared_experts, a.shared_intermediate_size)
                if mlp.shared_expert_gate is not None:
                    yield ParamSpec(p + "mlp.shared_expert_gate.weight", (1, H), _copy(mlp.shared_expert_gate))

    def _linear_attn_specs(self, p: str, la: GatedDeltaNet) -> Iterator[ParamSpec]:
        H = self.arch.hidden_size
        yield ParamSpec(p + "in_proj_qkvz.weight", (2 * la.key_dim + 2 * la.value_dim, H), la.set_in_proj_qkvz)
        yield ParamSpec(p + "in_proj_ba.weight", (2 * la.nv, H), la.set_in_proj_ba)
        yield ParamSpec(p + "conv1d.weight", (la.conv_dim, 1, la.K),
                        lambda t, _w=la.conv_weight: _w.data.copy_(t.reshape(_w.shape).to(_w.device, _w.dtype)))
        yield ParamSpec(p + "dt_bias", (la.nv,), _copy(la.dt_bias), "ones")
        yield ParamSpec(p + "A_log", (la.nv,), _copy(la.A_log), "zeros")
        yield ParamSpec(p + "norm.weight", (la.dv,), _copy(la.norm_weight), "ones")
        yield ParamSpec(p + "out_proj.weight", (H, la.value_dim), _copy(la.out_proj))

    def _gated_attn_specs(self, p: str, at: GatedGQAAttention) -> Iterator[ParamSpec]:
        H = self.arch.hidden_size
        nq, nkv, d = at.nq, at.nkv, at.d
        base = 2 * nq * d
        yield ParamSpec(p + "q_proj.weight", (2 * nq * d, H), at.set_q_proj)
        yield ParamSpec(p + "k_proj.weight", (nkv * d, H), _rows(at.qkv_proj, base, base + nkv * d))
        yield ParamSpec(p + "v_proj.weight", (nkv * d, H), _rows(at.qkv_proj, base + nkv * d, base + 2 * nkv * d))
        yield ParamSpec(p + "q_norm.weight", (d,), _copy_plus_one(at.q_norm.weight), "zeros")
        yield ParamSpec(p + "k_norm.weight", (d,), _copy_plus_one(at.k_norm.weight), "zeros")
        yield ParamSpec(p + "o_proj.weight", (H, nq * d), _copy(at.o_proj))


class AFDQwen3NextForCausalLM(AFDQwen3_5MoeForCausalLM):
    pass


__all__ = [
    "AFDCausalLM",
    "AFDDeepseekForCausalLM",
    "AFDDeepseekV2ForCausalLM",
    "AFDDeepseekV3ForCausalLM",
    "AFDDeepseekV4ForCausalLM",
    "AFDGlmMoeDsaForCausalLM",
    "AFDQwen3MoeForCausalLM",
    "AFDQwen3NextForCausalLM",
    "AFDQwen3_5MoeForCausalLM",
    "ParamSpec",
    "ROLES",
    "weight_roles",
]
