"""Checkpoint loading: role-filtered HF safetensors or seeded random init.

A checkpoint is streamed once; each tensor is kept only when the process's
AFD role needs it (:func:`afd_plugin_b200.models.model.weight_roles`, the same
split as the reference's ``_iter_role_weights``) and, for expert tensors, when
the expert lives on this expert-parallel shard.  fp8 block-scaled checkpoints
(``weight`` + ``weight_scale_inv``) load without dequantisation into the fp8
expert and MLP weights; fp8 tensors of parameters kept in the model dtype
(DeepSeek-V3's attention projections, for one) are dequantised with their
block scales on the way in.
"""

from __future__ import annotations

import glob
import json
import os
from collections.abc import Iterable, Iterator

import torch

from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.models.model import AFDCausalLM, weight_roles


def read_hf_config(path: str) -> ModelArchConfig:
    with open(os.path.join(path, "config.json")) as fh:
        return ModelArchConfig.from_hf_config(json.load(fh))


def iter_safetensors(path: str) -> Iterator[tuple[str, torch.Tensor]]:
    from safetensors import safe_open  # provided by the transformers install

    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors under {path}")
    for f in files:
        with safe_open(f, framework="pt", device="cpu") as fh:
            for name in fh.keys():
                yield name, fh.get_tensor(name)


def checkpoint_name(name: str) -> str | None:
    """The name a checkpoint tensor is loaded under, or None when no role loads it.

    Multimodal Qwen3.5 / 3.6 checkpoints keep the text model under
    ``model.language_model.``; their vision tower (``visual``) and
    multi-token-prediction head (``mtp``) are not served (the reference's
    Qwen3.5 wrapper gives those paths no role, ``qwen3_5.py:46-52``).
    """
    parts = name.split(".")
    if "visual" in parts or "mtp" in parts:
        return None
    if name.startswith("model.language_model."):
        return "model." + name[len("model.language_model."):]
    return name


def iter_role_weights(
    weights: Iterable[tuple[str, torch.Tensor]], *, role: str, arch: ModelArchConfig, compute_gate_on_attention: bool,
    route_on_attention: bool = False,
) -> Iterator[tuple[str, torch.Tensor]]:
    for raw, t in weights:
        name = checkpoint_name(raw)
        if name is None:
            continue
        if role == "colocated" or role in weight_roles(name, arch, compute_gate_on_attention=compute_gate_on_attention,
                                                       route_on_attention=route_on_attention):
            yield name, t


def load_weights(model: AFDCausalLM, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
    """Load ``(name, tensor)`` pairs into ``model``; returns the names consumed.

    Raises if a parameter this role owns is missing from the stream.
    """
    specs = {s.name: s for s in model.param_specs()}
    scale_of = {s.fp8_scale_name: s for s in specs.values() if s.fp8_scale_name}
    pending_scales: dict[str, torch.Tensor] = {}
    # fp8 checkpoint tensors whose parameter is not kept in fp8 (attention projections,
    # gates, ...): dequantised with their ``weight_scale_inv`` block scales once both are seen
    fp8_plain: dict[str, torch.Tensor] = {}
    plain_scales: dict[str, torch.Tensor] = {}
    loaded: set[str] = set()
    stream = iter_role_weights(
        weights, role=model.role, arch=model.arch, compute_gate_on_attention=model.compute_gate_on_attention,
        route_on_attention=getattr(model, "route_on_attention", False),
    )
    block = tuple(model.arch.weight_block_size)
    for name, t in stream:
        if name in specs:
            spec = specs[name]
            if t.dtype == torch.float8_e4m3fn and not spec.fp8_scale_name:
                fp8_plain[name] = t
                loaded.add(name)
                continue
            if t.dtype == torch.float8_e4m3fn and spec.fp8_scale_name:
                pending_scales.setdefault(spec.fp8_scale_name, None)  # type: ignore[arg-type]
            spec.setter(t)
            loaded.add(name)
        elif name in scale_of:
            pending_scales[name] = t
            loaded.add(name)
        elif name.endswith("_scale_inv") and name[: -len("_scale_inv")] in specs:
            plain_scales[name[: -len("_scale_inv")]] = t
    for name, t in fp8_plain.items():
        scale = plain_scales.get(name)
        if scale is None:
            raise ValueError(f"fp8 checkpoint tensor {name} has no {name}_scale_inv")
        from afd_plugin_b200.ops.reference import dequant_block

        specs[name].setter(dequant_block(t, scale.float(), block))
    # Block scales of pre-quantised checkpoints go into the scale slices.
    for sname, st in pending_scales.items():
        if st is None:
            raise ValueError(f"fp8 checkpoint is missing {sname}")
        _set_scale(model, scale_of[sname], st)
    missing = sorted(set(specs) - loaded)
    if missing:
        raise ValueError(f"checkpoint lacks {len(missing)} tensors for role {model.role!r}, e.g. {missing[:3]}")
    return loaded


def _set_scale(model: AFDCausalLM, spec, scale: torch.Tensor) -> None:
    # The spec's setter closes over the scale tensor; locate it through the name.
    name = spec.name
    parts = name.split(".")
    layer = model.layers[int(parts[2])]
    mlp = layer.mlp
    proj = parts[-2]
    if ".experts." in name:
        e = int(parts[5]) - mlp.experts.offset
        s13, s2 = mlp.experts.w13_scale[e], mlp.experts.w2_scale[e]
        inter = model.arch.moe_intermediate_size
    else:
        target = mlp.shared_experts if ".shared_experts." in name else mlp
        s13, s2 = target.w13_scale, target.w2_scale
        inter = target.w2.shape[1]
    if proj == "gate_proj":
        s13.data[: inter // 128].copy_(scale)
    elif proj == "up_proj":
        s13.data[inter // 128 :].copy_(scale)
    else:
        s2.data.copy_(scale)


def load_checkpoint(model: AFDCausalLM, path: str) -> set[str]:
    return load_weights(model, iter_safetensors(path))


__all__ = ["iter_role_weights", "iter_safetensors", "load_checkpoint", "load_weights", "read_hf_config"]
