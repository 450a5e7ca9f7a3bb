"""Architecture descriptions for the supported model families.

One dataclass covers the DeepSeek family (MLA attention, DeepSeek MoE with
shared experts, dense-first layers, optional grouped / biased routing, fp8
block-scaled weights) and the Qwen3-MoE family (GQA with QK-RMSNorm, routed
experts only).  ``from_hf_config`` reads a HuggingFace ``config.json`` dict;
the presets are the shapes the benchmarks name.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field, replace
from typing import Any

DEEPSEEK_ARCHS = ("DeepseekForCausalLM", "DeepseekV2ForCausalLM", "DeepseekV3ForCausalLM", "GlmMoeDsaForCausalLM")
QWEN3_MOE_ARCHS = ("Qwen3MoeForCausalLM",)
DEEPSEEK_V4_ARCHS = ("DeepseekV4ForCausalLM",)
QWEN3_5_ARCHS = ("Qwen3NextForCausalLM", "Qwen3_5MoeForCausalLM", "Qwen3_5MoeForConditionalGeneration")


@dataclass(frozen=True)
class ModelArchConfig:
    architecture: str
    hidden_size: int
    num_hidden_layers: int
    vocab_size: int
    num_attention_heads: int
    attention_type: str  # "mla" | "gqa"
    # MLA
    q_lora_rank: int | None = None
    kv_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    # DeepSeek sparse attention (DeepSeek-V3.2, GLM-MoE-DSA): a lightning
    # indexer scores every cached token and each query attends to its
    # ``index_topk`` best ones.  0 = dense MLA.
    index_topk: int = 0
    index_n_heads: int = 0
    index_head_dim: int = 0
    # GQA
    num_key_value_heads: int = 0
    head_dim: int = 0
    qk_norm: bool = False
    # FFN
    intermediate_size: int = 0
    first_k_dense_replace: int = 0
    moe_layer_freq: int = 1
    n_routed_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    n_shared_experts: int = 0
    scoring_func: str = "softmax"  # "softmax" | "sigmoid"
    topk_method: str = "greedy"  # "greedy" | "group_limited_greedy" | "noaux_tc"
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0
    # misc
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: dict | None = None
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    # Hybrid linear attention (Qwen3.5 / Qwen3-Next): per-layer kinds and the
    # Gated DeltaNet shapes.  ``layer_types`` None means every layer is full attention.
    layer_types: tuple[str, ...] | None = None
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel_dim: int = 4
    partial_rotary_factor: float = 1.0
    attn_output_gate: bool = False  # full attention: output * sigmoid(gate half of q_proj)
    shared_expert_intermediate_size: int = 0  # overrides n_shared_experts * moe_intermediate_size
    shared_expert_gate: bool = False  # shared expert output * sigmoid(x . w)
    norm_offset_one: bool = False  # checkpoint RMSNorm weights are stored as (w - 1)
    # DeepSeek-V4: manifold-constrained hyper-connections (hc_mult residual
    # streams) and hash routing (expert ids from a token-id table) in the first
    # num_hash_layers MoE layers.
    hc_mult: int = 0
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    num_hash_layers: int = 0
    # End-of-sequence token ids: generation stops there unless a request ignores EOS.
    eos_token_id: tuple[int, ...] = ()
    # "fp8_block": e4m3 weights with 128x128 scales for experts and dense MLPs.
    quant: str | None = None
    weight_block_size: tuple[int, int] = (128, 128)
    extra: dict = field(default_factory=dict)

    # -------------------------------------------------------------- helpers
    @property
    def is_mla(self) -> bool:
        return self.attention_type == "mla"

    def is_moe_layer(self, layer_idx: int) -> bool:
        return (
            self.n_routed_experts > 0
            and layer_idx >= self.first_k_dense_replace
            and layer_idx % max(1, self.moe_layer_freq) == 0
        )

    @property
    def moe_layer_indices(self) -> tuple[int, ...]:
        return tuple(i for i in range(self.num_hidden_layers) if self.is_moe_layer(i))

    @property
    def has_indexer(self) -> bool:
        return self.is_mla and self.index_topk > 0

    @property
    def qk_head_dim(self) -> int:
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def kv_cache_width(self) -> int:
        """Elements cached per token per layer (MLA: latent+rope; GQA: K and V)."""
        if self.is_mla:
            return self.kv_lora_rank + self.qk_rope_head_dim + (self.index_head_dim if self.has_indexer else 0)
        return 2 * self.num_key_value_heads * self.head_dim

    @property
    def softmax_scale(self) -> float:
        if self.is_mla:
            scale = 1.0 / math.sqrt(self.qk_head_dim)
            rs = self.rope_scaling or {}
            if rs.get("type", rs.get("rope_type")) in ("yarn", "deepseek_yarn"):
                mscale_all = float(rs.get("mscale_all_dim", 0.0) or 0.0)
                factor = float(rs.get("factor", 1.0))
                if mscale_all:
                    m = yarn_get_mscale(factor, mscale_all)
                    scale = scale * m * m
            return scale
        return 1.0 / math.sqrt(self.head_dim)

    @property
    def shared_intermediate_size(self) -> int:
        if self.shared_expert_intermediate_size:
            return self.shared_expert_intermediate_size
        return self.moe_intermediate_size * self.n_shared_experts

    @property
    def has_shared_experts(self) -> bool:
        return self.shared_intermediate_size > 0

    def is_linear_attention_layer(self, layer_idx: int) -> bool:
        return self.layer_types is not None and self.layer_types[layer_idx] == "linear_attention"

    @property
    def linear_attention_layers(self) -> tuple[int, ...]:
        return tuple(i for i in range(self.num_hidden_layers) if self.is_linear_attention_layer(i))

    @property
    def full_attention_layers(self) -> tuple[int, ...]:
        return tuple(i for i in range(self.num_hidden_layers) if not self.is_linear_attention_layer(i))

    @property
    def rotary_dim(self) -> int:
        if self.is_mla:
            return self.qk_rope_head_dim
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def linear_key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def linear_value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def linear_conv_dim(self) -> int:
        return 2 * self.linear_key_dim + self.linear_value_dim

    def scaled(self, **overrides: Any) -> "ModelArchConfig":
        return replace(self, **overrides)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["weight_block_size"] = list(self.weight_block_size)
        return d

    # -------------------------------------------------------------- parsing
    @classmethod
    def from_hf_config(cls, hf: dict) -> "ModelArchConfig":
        text = hf.get("text_config")
        if isinstance(text, dict) and "hidden_size" not in hf:
            # multimodal wrappers (Qwen3.5 / 3.6 ConditionalGeneration) keep the
            # language model's fields under text_config
            hf = {**text, "architectures": hf.get("architectures") or text.get("architectures"),
                  "quantization_config": hf.get("quantization_config") or text.get("quantization_config"),
                  "eos_token_id": hf.get("eos_token_id", text.get("eos_token_id"))}
        cfg = cls._parse_hf(hf)
        eos = hf.get("eos_token_id", (hf.get("text_config") or {}).get("eos_token_id"))
        ids = tuple(int(e) for e in (eos if isinstance(eos, (list, tuple)) else [eos]) if e is not None)
        return replace(cfg, eos_token_id=ids) if ids else cfg

    @classmethod
    def _parse_hf(cls, hf: dict) -> "ModelArchConfig":
        archs = hf.get("architectures") or [""]
        arch = archs[0]
        if arch.startswith("AFD"):
            arch = arch[3:]
        quant = None
        block = (128, 128)
        qc = hf.get("quantization_config") or {}
        if qc.get("quant_method") == "fp8":
            quant = "fp8_block"
            block = tuple(qc.get("weight_block_size", [128, 128]))
        if arch in DEEPSEEK_V4_ARCHS or hf.get("model_type") == "deepseek_v4":
            return cls(
                architecture="DeepseekV4ForCausalLM",
                hidden_size=hf["hidden_size"],
                num_hidden_layers=hf["num_hidden_layers"],
                vocab_size=hf["vocab_size"],
                num_attention_heads=hf["num_attention_heads"],
                attention_type="mla",
                q_lora_rank=hf.get("q_lora_rank"),
                kv_lora_rank=hf["kv_lora_rank"],
                qk_nope_head_dim=hf["qk_nope_head_dim"],
                qk_rope_head_dim=hf["qk_rope_head_dim"],
                v_head_dim=hf["v_head_dim"],
                intermediate_size=hf.get("intermediate_size", 0),
                first_k_dense_replace=hf.get("first_k_dense_replace", 0),
                n_routed_experts=hf["n_routed_experts"],
                num_experts_per_tok=hf["num_experts_per_tok"],
                moe_intermediate_size=hf["moe_intermediate_size"],
                n_shared_experts=hf.get("n_shared_experts") or 0,
                scoring_func=hf.get("scoring_func", "sqrtsoftplus"),
                topk_method=hf.get("topk_method", "noaux_tc"),
                n_group=hf.get("n_group") or 1,
                topk_group=hf.get("topk_group") or 1,
                norm_topk_prob=bool(hf.get("norm_topk_prob", True)),
                routed_scaling_factor=float(hf.get("routed_scaling_factor", 1.5)),
                rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
                rope_theta=hf.get("rope_theta", 10000.0),
                rope_scaling=hf.get("rope_scaling"),
                max_position_embeddings=hf.get("max_position_embeddings", 65536),
                hc_mult=hf["hc_mult"],
                hc_sinkhorn_iters=hf.get("hc_sinkhorn_iters", 20),
                hc_eps=hf.get("hc_eps", 1e-6),
                num_hash_layers=hf.get("num_hash_layers", 0),
                quant=quant,
                weight_block_size=block,
            )
        if (arch == "DeepseekForCausalLM" or hf.get("model_type") == "deepseek") and "kv_lora_rank" not in hf:
            # DeepSeek V1 (DeepSeekMoE): multi-head attention, fine-grained + shared experts
            heads = hf["num_attention_heads"]
            return cls(
                architecture="DeepseekForCausalLM",
                hidden_size=hf["hidden_size"],
                num_hidden_layers=hf["num_hidden_layers"],
                vocab_size=hf["vocab_size"],
                num_attention_heads=heads,
                attention_type="gqa",
                num_key_value_heads=hf.get("num_key_value_heads") or heads,
                head_dim=hf.get("head_dim") or hf["hidden_size"] // heads,
                qk_norm=False,
                intermediate_size=hf["intermediate_size"],
                first_k_dense_replace=hf.get("first_k_dense_replace", 0),
                moe_layer_freq=hf.get("moe_layer_freq", 1),
                n_routed_experts=hf.get("n_routed_experts") or 0,
                num_experts_per_tok=hf.get("num_experts_per_tok") or 0,
                moe_intermediate_size=hf.get("moe_intermediate_size", 0),
                n_shared_experts=hf.get("n_shared_experts") or 0,
                scoring_func=hf.get("scoring_func", "softmax"),
                norm_topk_prob=bool(hf.get("norm_topk_prob", False)),
                rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
                rope_theta=hf.get("rope_theta", 10000.0),
                rope_scaling=hf.get("rope_scaling"),
                max_position_embeddings=hf.get("max_position_embeddings", 4096),
                tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
                quant=quant,
                weight_block_size=block,
            )
        if arch in DEEPSEEK_ARCHS or hf.get("model_type", "").startswith("deepseek"):
            return cls(
                architecture=arch or "DeepseekV2ForCausalLM",
                hidden_size=hf["hidden_size"],
                num_hidden_layers=hf["num_hidden_layers"],
                vocab_size=hf["vocab_size"],
                num_attention_heads=hf["num_attention_heads"],
                attention_type="mla",
                q_lora_rank=hf.get("q_lora_rank"),
                kv_lora_rank=hf["kv_lora_rank"],
                qk_nope_head_dim=hf["qk_nope_head_dim"],
                qk_rope_head_dim=hf["qk_rope_head_dim"],
                v_head_dim=hf["v_head_dim"],
                intermediate_size=hf["intermediate_size"],
                first_k_dense_replace=hf.get("first_k_dense_replace", 0),
                moe_layer_freq=hf.get("moe_layer_freq", 1),
                n_routed_experts=hf.get("n_routed_experts") or 0,
                num_experts_per_tok=hf.get("num_experts_per_tok") or 0,
                moe_intermediate_size=hf.get("moe_intermediate_size", 0),
                n_shared_experts=hf.get("n_shared_experts") or 0,
                scoring_func=hf.get("scoring_func", "softmax"),
                topk_method=hf.get("topk_method", "greedy"),
                n_group=hf.get("n_group") or 1,
                topk_group=hf.get("topk_group") or 1,
                norm_topk_prob=bool(hf.get("norm_topk_prob", False)),
                routed_scaling_factor=float(hf.get("routed_scaling_factor", 1.0)),
                rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
                rope_theta=hf.get("rope_theta", 10000.0),
                rope_scaling=hf.get("rope_scaling"),
                max_position_embeddings=hf.get("max_position_embeddings", 4096),
                tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
                index_topk=int(hf.get("index_topk") or 0),
                index_n_heads=int(hf.get("index_n_heads") or 0),
                index_head_dim=int(hf.get("index_head_dim") or 0),
                quant=quant,
                weight_block_size=block,
            )
        if arch in QWEN3_MOE_ARCHS or hf.get("model_type") == "qwen3_moe":
            mlp_only = hf.get("mlp_only_layers") or []
            if mlp_only:
                raise ValueError("Qwen3-MoE mlp_only_layers are not supported")
            return cls(
                architecture="Qwen3MoeForCausalLM",
                hidden_size=hf["hidden_size"],
                num_hidden_layers=hf["num_hidden_layers"],
                vocab_size=hf["vocab_size"],
                num_attention_heads=hf["num_attention_heads"],
                attention_type="gqa",
                num_key_value_heads=hf["num_key_value_heads"],
                head_dim=hf.get("head_dim") or hf["hidden_size"] // hf["num_attention_heads"],
                qk_norm=True,
                intermediate_size=hf.get("intermediate_size", 0),
                first_k_dense_replace=0,
                moe_layer_freq=hf.get("decoder_sparse_step", 1),
                n_routed_experts=hf["num_experts"],
                num_experts_per_tok=hf["num_experts_per_tok"],
                moe_intermediate_size=hf["moe_intermediate_size"],
                n_shared_experts=0,
                norm_topk_prob=bool(hf.get("norm_topk_prob", True)),
                rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
                rope_theta=hf.get("rope_theta", 1000000.0),
                rope_scaling=hf.get("rope_scaling"),
                max_position_embeddings=hf.get("max_position_embeddings", 40960),
                tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
                quant=quant,
                weight_block_size=block,
            )
        if arch in QWEN3_5_ARCHS or hf.get("model_type") in ("qwen3_next", "qwen3_5_moe", "qwen3_5_moe_text"):
            L = hf["num_hidden_layers"]
            types = hf.get("layer_types")
            if types is None:
                interval = hf.get("full_attention_interval", 4)
                types = ["full_attention" if (i + 1) % interval == 0 else "linear_attention" for i in range(L)]
            if hf.get("mlp_only_layers"):
                raise ValueError("Qwen3.5 mlp_only_layers are not supported")
            return cls(
                architecture=arch if arch in QWEN3_5_ARCHS else "Qwen3NextForCausalLM",
                hidden_size=hf["hidden_size"],
                num_hidden_layers=L,
                vocab_size=hf["vocab_size"],
                num_attention_heads=hf["num_attention_heads"],
                attention_type="gqa",
                num_key_value_heads=hf["num_key_value_heads"],
                head_dim=hf.get("head_dim") or hf["hidden_size"] // hf["num_attention_heads"],
                qk_norm=True,
                intermediate_size=hf.get("intermediate_size", 0),
                moe_layer_freq=hf.get("decoder_sparse_step", 1),
                n_routed_experts=hf["num_experts"],
                num_experts_per_tok=hf["num_experts_per_tok"],
                moe_intermediate_size=hf["moe_intermediate_size"],
                shared_expert_intermediate_size=hf.get("shared_expert_intermediate_size", 0),
                shared_expert_gate=bool(hf.get("shared_expert_intermediate_size", 0)),
                norm_topk_prob=bool(hf.get("norm_topk_prob", True)),
                rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
                rope_theta=hf.get("rope_theta", 10000000.0),
                rope_scaling=hf.get("rope_scaling"),
                max_position_embeddings=hf.get("max_position_embeddings", 262144),
                tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
                layer_types=tuple(types),
                linear_num_key_heads=hf["linear_num_key_heads"],
                linear_num_value_heads=hf["linear_num_value_heads"],
                linear_key_head_dim=hf["linear_key_head_dim"],
                linear_value_head_dim=hf["linear_value_head_dim"],
                linear_conv_kernel_dim=hf.get("linear_conv_kernel_dim", 4),
                partial_rotary_factor=float(hf.get("partial_rotary_factor", 0.25)),
                attn_output_gate=True,
                norm_offset_one=True,
                quant=quant,
                weight_block_size=block,
            )
        raise ValueError(f"unsupported architecture {arch!r}")


def yarn_get_mscale(scale: float, mscale: float = 1.0) -> float:
    if scale <= 1.0:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


# ---------------------------------------------------------------------------
# Presets named by the benchmark configurations.
# ---------------------------------------------------------------------------

TINY_DSV2 = ModelArchConfig(
    architecture="DeepseekV2ForCausalLM",
    hidden_size=256,
    num_hidden_layers=2,
    vocab_size=1024,
    num_attention_heads=4,
    attention_type="mla",
    q_lora_rank=None,
    kv_lora_rank=64,
    qk_nope_head_dim=32,
    qk_rope_head_dim=32,
    v_head_dim=32,
    intermediate_size=512,
    first_k_dense_replace=1,
    n_routed_experts=8,
    num_experts_per_tok=2,
    moe_intermediate_size=128,
    n_shared_experts=1,
    scoring_func="softmax",
    topk_method="greedy",
    max_position_embeddings=2048,
)

DSV2_LITE = ModelArchConfig(
    architecture="DeepseekV2ForCausalLM",
    hidden_size=2048,
    num_hidden_layers=27,
    vocab_size=102400,
    num_attention_heads=16,
    attention_type="mla",
    q_lora_rank=None,
    kv_lora_rank=512,
    qk_nope_head_dim=128,
    qk_rope_head_dim=64,
    v_head_dim=128,
    intermediate_size=10944,
    first_k_dense_replace=1,
    n_routed_experts=64,
    num_experts_per_tok=6,
    moe_intermediate_size=1408,
    n_shared_experts=2,
    scoring_func="softmax",
    topk_method="greedy",
    norm_topk_prob=False,
    routed_scaling_factor=1.0,
    rms_norm_eps=1e-6,
    rope_theta=10000.0,
    rope_scaling={
        "type": "yarn",
        "factor": 40,
        "beta_fast": 32,
        "beta_slow": 1,
        "mscale": 0.707,
        "mscale_all_dim": 0.707,
        "original_max_position_embeddings": 4096,
    },
    max_position_embeddings=163840,
)

QWEN3_30B_A3B = ModelArchConfig(
    architecture="Qwen3MoeForCausalLM",
    hidden_size=2048,
    num_hidden_layers=48,
    vocab_size=151936,
    num_attention_heads=32,
    attention_type="gqa",
    num_key_value_heads=4,
    head_dim=128,
    qk_norm=True,
    intermediate_size=6144,
    n_routed_experts=128,
    num_experts_per_tok=8,
    moe_intermediate_size=768,
    n_shared_experts=0,
    norm_topk_prob=True,
    rms_norm_eps=1e-6,
    rope_theta=1000000.0,
    max_position_embeddings=40960,
)

DSV3_32L = ModelArchConfig(
    architecture="DeepseekV3ForCausalLM",
    hidden_size=7168,
    num_hidden_layers=32,
    vocab_size=129280,
    num_attention_heads=128,
    attention_type="mla",
    q_lora_rank=1536,
    kv_lora_rank=512,
    qk_nope_head_dim=128,
    qk_rope_head_dim=64,
    v_head_dim=128,
    intermediate_size=18432,
    first_k_dense_replace=3,
    n_routed_experts=256,
    num_experts_per_tok=8,
    moe_intermediate_size=2048,
    n_shared_experts=1,
    scoring_func="sigmoid",
    topk_method="noaux_tc",
    n_group=8,
    topk_group=4,
    norm_topk_prob=True,
    routed_scaling_factor=2.5,
    rms_norm_eps=1e-6,
    rope_theta=10000.0,
    rope_scaling={
        "type": "yarn",
        "factor": 40,
        "beta_fast": 32,
        "beta_slow": 1,
        "mscale": 1.0,
        "mscale_all_dim": 1.0,
        "original_max_position_embeddings": 4096,
    },
    max_position_embeddings=163840,
    quant="fp8_block",
)

TINY_QWEN3_MOE = ModelArchConfig(
    architecture="Qwen3MoeForCausalLM",
    hidden_size=256,
    num_hidden_layers=2,
    vocab_size=1024,
    num_attention_heads=4,
    attention_type="gqa",
    num_key_value_heads=2,
    head_dim=64,
    qk_norm=True,
    n_routed_experts=8,
    num_experts_per_tok=2,
    moe_intermediate_size=128,
    norm_topk_prob=True,
    rope_theta=1000000.0,
    max_position_embeddings=2048,
)

TINY_DSV3 = DSV3_32L.scaled(
    hidden_size=256,
    num_hidden_layers=3,
    vocab_size=1024,
    num_attention_heads=4,
    q_lora_rank=64,
    kv_lora_rank=64,
    qk_nope_head_dim=32,
    qk_rope_head_dim=32,
    v_head_dim=32,
    intermediate_size=512,
    first_k_dense_replace=1,
    n_routed_experts=16,
    num_experts_per_tok=4,
    moe_intermediate_size=128,
    n_group=4,
    topk_group=2,
    max_position_embeddings=2048,
    quant=None,
)

# DeepSeek V1 (deepseek-moe-16b): multi-head attention (16 x 128), 64
# fine-grained experts top-6 plus 2 shared experts, layer 0 dense.
DSV1_MOE_16B = ModelArchConfig(
    architecture="DeepseekForCausalLM",
    hidden_size=2048,
    num_hidden_layers=28,
    vocab_size=102400,
    num_attention_heads=16,
    attention_type="gqa",
    num_key_value_heads=16,
    head_dim=128,
    intermediate_size=10944,
    first_k_dense_replace=1,
    n_routed_experts=64,
    num_experts_per_tok=6,
    moe_intermediate_size=1408,
    n_shared_experts=2,
    max_position_embeddings=4096,
)

TINY_DSV1 = DSV1_MOE_16B.scaled(
    hidden_size=256,
    num_hidden_layers=3,
    vocab_size=1024,
    num_attention_heads=4,
    num_key_value_heads=4,
    head_dim=64,
    intermediate_size=512,
    n_routed_experts=8,
    num_experts_per_tok=2,
    moe_intermediate_size=128,
    n_shared_experts=1,
    max_position_embeddings=2048,
)

# DeepSeek-V3.2 shapes on the 32-layer DSV3 body: DeepSeek sparse attention
# with a 64-head, 128-dim lightning indexer selecting 2048 tokens per query.
DSV32_32L = DSV3_32L.scaled(architecture="DeepseekV32ForCausalLM", index_topk=2048, index_n_heads=64,
                            index_head_dim=128)

# Tiny DeepSeek-V3.2: the indexer keeps 8 tokens, so prompts of a few dozen
# tokens exercise the sparse path.
TINY_DSV32 = TINY_DSV3.scaled(architecture="DeepseekV32ForCausalLM", index_topk=8, index_n_heads=4,
                              index_head_dim=48)

# Tiny DeepSeek with the production MLA shapes (latent 512 + rope 64, 16
# heads), so GPU tests exercise the specialised decode kernel.
TINY_DSV2_MLA512 = TINY_DSV2.scaled(
    kv_lora_rank=512, qk_rope_head_dim=64, qk_nope_head_dim=128, v_head_dim=128, num_attention_heads=16
)

# Qwen3-Next-80B-A3B shapes (the published config of the Qwen3.5 / Qwen3-Next
# hybrid family): 48 layers, every 4th full attention, 512 experts top-10.
QWEN3_NEXT_80B_A3B = ModelArchConfig(
    architecture="Qwen3NextForCausalLM",
    hidden_size=2048,
    num_hidden_layers=48,
    vocab_size=151936,
    num_attention_heads=16,
    attention_type="gqa",
    num_key_value_heads=2,
    head_dim=256,
    qk_norm=True,
    intermediate_size=5120,
    n_routed_experts=512,
    num_experts_per_tok=10,
    moe_intermediate_size=512,
    shared_expert_intermediate_size=512,
    shared_expert_gate=True,
    norm_topk_prob=True,
    rms_norm_eps=1e-6,
    rope_theta=10000000.0,
    max_position_embeddings=262144,
    layer_types=tuple("full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(48)),
    linear_num_key_heads=16,
    linear_num_value_heads=32,
    linear_key_head_dim=128,
    linear_value_head_dim=128,
    linear_conv_kernel_dim=4,
    partial_rotary_factor=0.25,
    attn_output_gate=True,
    norm_offset_one=True,
)

TINY_QWEN3_5 = QWEN3_NEXT_80B_A3B.scaled(
    architecture="Qwen3_5MoeForCausalLM",
    hidden_size=256,
    num_hidden_layers=4,
    vocab_size=1024,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=64,
    n_routed_experts=8,
    num_experts_per_tok=2,
    moe_intermediate_size=128,
    shared_expert_intermediate_size=128,
    max_position_embeddings=2048,
    layer_types=("linear_attention", "linear_attention", "linear_attention", "full_attention"),
    linear_num_key_heads=2,
    linear_num_value_heads=4,
    linear_key_head_dim=32,
    linear_value_head_dim=32,
)


# DeepSeek-V4-style test shapes: MLA attention, 4 mHC residual streams, hash
# routing in the first MoE layer, sqrt-softplus scoring with a selection bias.
TINY_DSV4 = ModelArchConfig(
    architecture="DeepseekV4ForCausalLM",
    hidden_size=256,
    num_hidden_layers=3,
    vocab_size=1024,
    num_attention_heads=4,
    attention_type="mla",
    q_lora_rank=64,
    kv_lora_rank=64,
    qk_nope_head_dim=32,
    qk_rope_head_dim=32,
    v_head_dim=32,
    intermediate_size=512,
    first_k_dense_replace=1,
    n_routed_experts=8,
    num_experts_per_tok=2,
    moe_intermediate_size=128,
    n_shared_experts=1,
    scoring_func="sqrtsoftplus",
    topk_method="noaux_tc",
    norm_topk_prob=True,
    routed_scaling_factor=1.5,
    max_position_embeddings=2048,
    hc_mult=4,
    hc_sinkhorn_iters=20,
    hc_eps=1e-6,
    num_hash_layers=2,
)


PRESETS: dict[str, ModelArchConfig] = {
    "tiny-dsv2-mla512": TINY_DSV2_MLA512,
    "tiny-dsv2": TINY_DSV2,
    "tiny-dsv3": TINY_DSV3,
    "tiny-dsv32": TINY_DSV32,
    "tiny-dsv1": TINY_DSV1,
    "deepseek-moe-16b": DSV1_MOE_16B,
    "deepseek-v3.2-32l": DSV32_32L,
    "tiny-qwen3-moe": TINY_QWEN3_MOE,
    "deepseek-v2-lite": DSV2_LITE,
    "qwen3-30b-a3b": QWEN3_30B_A3B,
    "deepseek-v3-32l": DSV3_32L,
    "tiny-qwen3.5": TINY_QWEN3_5,
    "tiny-dsv4": TINY_DSV4,
    "qwen3-next-80b-a3b": QWEN3_NEXT_80B_A3B,
}


def get_preset(name: str) -> ModelArchConfig:
    try:
        return PRESETS[name]
    except KeyError:
        raise ValueError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}") from None


__all__ = [
    "DSV2_LITE",
    "DSV1_MOE_16B",
    "DSV32_32L",
    "DSV3_32L",
    "ModelArchConfig",
    "PRESETS",
    "QWEN3_30B_A3B",
    "QWEN3_NEXT_80B_A3B",
    "TINY_QWEN3_5",
    "TINY_DSV2",
    "TINY_DSV3",
    "TINY_DSV4",
    "TINY_QWEN3_MOE",
    "get_preset",
    "yarn_get_mscale",
]
