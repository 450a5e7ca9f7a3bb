"""Model zoo: role-aware AFD wrappers, architecture presets and loading.

``MODEL_REGISTRY`` maps HF architecture names (and their ``AFD``-prefixed
aliases, as registered by the reference in ``afd_plugin/__init__.py:97-140``)
to wrapper classes.
"""

from __future__ import annotations

import torch

from afd_plugin_b200.models.configs import PRESETS, ModelArchConfig, get_preset
from afd_plugin_b200.models.layers import AttentionMetadata
from afd_plugin_b200.models.model import (
    AFDCausalLM,
    AFDDeepseekForCausalLM,
    AFDDeepseekV2ForCausalLM,
    AFDDeepseekV3ForCausalLM,
    AFDDeepseekV4ForCausalLM,
    AFDGlmMoeDsaForCausalLM,
    AFDQwen3MoeForCausalLM,
    AFDQwen3NextForCausalLM,
    AFDQwen3_5MoeForCausalLM,
    weight_roles,
)

MODEL_REGISTRY: dict[str, type[AFDCausalLM]] = {
    "DeepseekForCausalLM": AFDDeepseekForCausalLM,
    "DeepseekV2ForCausalLM": AFDDeepseekV2ForCausalLM,
    "DeepseekV3ForCausalLM": AFDDeepseekV3ForCausalLM,
    "DeepseekV32ForCausalLM": AFDDeepseekV3ForCausalLM,
    "DeepseekV4ForCausalLM": AFDDeepseekV4ForCausalLM,
    "GlmMoeDsaForCausalLM": AFDGlmMoeDsaForCausalLM,
    "Qwen3MoeForCausalLM": AFDQwen3MoeForCausalLM,
    "Qwen3NextForCausalLM": AFDQwen3NextForCausalLM,
    "Qwen3_5MoeForCausalLM": AFDQwen3_5MoeForCausalLM,
    "Qwen3_5MoeForConditionalGeneration": AFDQwen3_5MoeForCausalLM,
}
MODEL_REGISTRY.update({"AFD" + k: v for k, v in list(MODEL_REGISTRY.items())})


def model_class_for(arch: ModelArchConfig) -> type[AFDCausalLM]:
    try:
        return MODEL_REGISTRY[arch.architecture]
    except KeyError:
        raise ValueError(f"no AFD wrapper for architecture {arch.architecture!r}") from None


def build_model(
    arch: ModelArchConfig,
    *,
    role: str = "colocated",
    dtype: torch.dtype = torch.bfloat16,
    device="cpu",
    compute_gate_on_attention: bool = False,
    ep_rank: int = 0,
    ep_size: int = 1,
    seed: int = 0,
    checkpoint: str | None = None,
    max_positions: int | None = None,
    route_on_attention: bool = False,
    init_on: str | None = None,
    tp=None,
) -> AFDCausalLM:
    """``tp`` (:class:`afd_plugin_b200.models.layers.TPInfo`) shards the attention heads."""
    cls = model_class_for(arch)
    kw = {} if tp is None else {"tp": tp}
    model = cls(
        arch,
        role=role,
        dtype=dtype,
        device=device,
        compute_gate_on_attention=compute_gate_on_attention,
        ep_rank=ep_rank,
        ep_size=ep_size,
        max_positions=max_positions,
        route_on_attention=route_on_attention,
        **kw,
    )
    if checkpoint is None:
        model.init_random(seed, generate_on=init_on)
    else:
        from afd_plugin_b200.models.loader import load_checkpoint

        load_checkpoint(model, checkpoint)
    model.finalize_weights()
    return model


__all__ = [
    "AFDCausalLM",
    "AttentionMetadata",
    "MODEL_REGISTRY",
    "ModelArchConfig",
    "PRESETS",
    "build_model",
    "get_preset",
    "model_class_for",
    "weight_roles",
]
