"""afd_plugin_b200: Attention-FFN Disaggregation serving for NVIDIA B200.

Entry points:

* :func:`register_afd` -- the ``vllm.general_plugins`` hook (also callable
  standalone): registers the ``AFD<Arch>`` model aliases and validates the
  environment.
* :class:`afd_plugin_b200.runtime.engine.LLMEngine` -- the standalone engine
  (with :class:`~afd_plugin_b200.runtime.sampling.SamplingParams`).
* :mod:`afd_plugin_b200.runtime.workers` -- Attention / FFN role workers.
* ``python -m afd_plugin_b200.serving`` -- the completions server;
  ``python -m afd_plugin_b200.serving.proxy`` -- the load-balancing and
  prefill/decode proxy; ``python -m afd_plugin_b200.e2e.runner`` -- scenario runs.
"""

from __future__ import annotations

import importlib
import logging
import os

__version__ = "0.1.0"
log = logging.getLogger(__name__)

_LAZY = {
    "AFDAttentionWorker": "afd_plugin_b200.runtime.workers",
    "AFDFFNWorker": "afd_plugin_b200.runtime.workers",
    "LLMEngine": "afd_plugin_b200.runtime.engine",
    "ModelRunner": "afd_plugin_b200.runtime.model_runner",
    "FFNModelRunner": "afd_plugin_b200.runtime.ffn_runner",
    "AFDConfig": "afd_plugin_b200.config",
    "EngineConfig": "afd_plugin_b200.engine_config",
    "SamplingParams": "afd_plugin_b200.runtime.sampling",
}

# HF architecture -> AFD alias (what ``register_afd`` publishes).
MODEL_ALIASES: dict[str, str] = {
    "DeepseekForCausalLM": "AFDDeepseekForCausalLM",
    "DeepseekV2ForCausalLM": "AFDDeepseekV2ForCausalLM",
    "DeepseekV3ForCausalLM": "AFDDeepseekV3ForCausalLM",
    "DeepseekV32ForCausalLM": "AFDDeepseekV32ForCausalLM",
    "DeepseekV4ForCausalLM": "AFDDeepseekV4ForCausalLM",
    "GlmMoeDsaForCausalLM": "AFDGlmMoeDsaForCausalLM",
    "Qwen3MoeForCausalLM": "AFDQwen3MoeForCausalLM",
    "Qwen3_5MoeForConditionalGeneration": "AFDQwen3_5MoeForConditionalGeneration",
    "Qwen3_5MoeForCausalLM": "AFDQwen3_5MoeForCausalLM",
    "Qwen3NextForCausalLM": "AFDQwen3NextForCausalLM",
}
# Aliases whose wrapper class carries another name.
_ALIAS_CLASS = {
    "AFDDeepseekV32ForCausalLM": "AFDDeepseekV3ForCausalLM",
    "AFDQwen3_5MoeForConditionalGeneration": "AFDQwen3_5MoeForCausalLM",
}

_REGISTERED = False


def __getattr__(name: str):
    if name in _LAZY:
        return getattr(importlib.import_module(_LAZY[name]), name)
    raise AttributeError(name)


def _force_spawn_multiprocessing_if_requested() -> None:
    if os.environ.get("AFD_FORCE_SPAWN_MULTIPROCESSING", "").lower() in ("1", "true", "yes", "on"):
        os.environ["VLLM_WORKER_MULTIPROC_METHOD"] = "spawn"
        import multiprocessing

        try:
            multiprocessing.set_start_method("spawn", force=False)
        except RuntimeError:
            pass


def register_afd() -> dict[str, str]:
    """Plugin hook (``vllm.general_plugins: afd = afd_plugin_b200:register_afd``).

    Registers every ``AFD<Arch>`` alias in this package's model registry; the
    models run on this package's own engine (``LLMEngine``, the Attention /
    FFN workers, ``python -m afd_plugin_b200.serving``), not inside a vLLM
    worker.  vLLM cannot instantiate these standalone modules, so its
    ``ModelRegistry`` receives the aliases (as lazy ``module:Class`` strings)
    only when ``AFD_PUBLISH_VLLM_ALIASES=1`` asks for it, e.g. for tooling that
    resolves architecture names.  Idempotent; returns the alias map.
    """
    global _REGISTERED
    _force_spawn_multiprocessing_if_requested()
    if _REGISTERED:
        return dict(MODEL_ALIASES)
    from afd_plugin_b200.models import MODEL_REGISTRY

    for arch, alias in MODEL_ALIASES.items():
        MODEL_REGISTRY.setdefault(alias, MODEL_REGISTRY[arch])
    if os.environ.get("AFD_PUBLISH_VLLM_ALIASES", "").lower() not in ("1", "true", "yes", "on"):
        _REGISTERED = True
        return dict(MODEL_ALIASES)
    from afd_plugin_b200.compat import can_publish_aliases

    if not can_publish_aliases():
        _REGISTERED = True
        return dict(MODEL_ALIASES)
    try:  # opt-in: publish the names into vLLM when present
        from vllm import ModelRegistry  # type: ignore

        supported = set(ModelRegistry.get_supported_archs())
        for alias in MODEL_ALIASES.values():
            if alias not in supported:
                ModelRegistry.register_model(alias, f"afd_plugin_b200.models.model:{_class_name(alias)}")
    except Exception as exc:  # noqa: BLE001 - vLLM is optional
        log.debug("vLLM registry not updated: %s", exc)
    _REGISTERED = True
    return dict(MODEL_ALIASES)


def _class_name(alias: str) -> str:
    return _ALIAS_CLASS.get(alias, alias)


__all__ = ["MODEL_ALIASES", "__version__", "register_afd", *_LAZY]
