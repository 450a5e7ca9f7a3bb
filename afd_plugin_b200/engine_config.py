"""Engine-level configuration objects for the standalone runtime.

Attribute names mirror the ones AFD code reads from vLLM's ``VllmConfig``
(``model_config.enforce_eager``, ``parallel_config.data_parallel_size``,
``compilation_config.cudagraph_mode``, ``additional_config["afd"]`` ...) so the
same policy helpers work on either object.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from afd_plugin_b200.models.configs import ModelArchConfig


@dataclass
class ModelConfig:
    arch: ModelArchConfig
    dtype: torch.dtype = torch.bfloat16
    enforce_eager: bool = False
    max_model_len: int = 4096
    seed: int = 0
    # Path to a HF checkpoint directory; ``None`` means seeded random init.
    checkpoint: str | None = None

    @property
    def hf_config(self) -> ModelArchConfig:
        return self.arch

    hf_text_config = hf_config


@dataclass
class ParallelConfig:
    data_parallel_size: int = 1
    data_parallel_rank: int = 0
    tensor_parallel_size: int = 1
    prefill_context_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    use_ubatching: bool = False
    num_ubatches: int = 1
    enable_eplb: bool = False
    use_sequence_parallel_moe: bool = False
    enable_expert_parallel: bool = True


@dataclass
class CompilationConfig:
    # ``None`` disables graphs; only ``FULL_DECODE_ONLY`` is accepted otherwise.
    cudagraph_mode: str | None = "FULL_DECODE_ONLY"
    cudagraph_capture_sizes: list[int] = field(default_factory=lambda: [64])


@dataclass
class CacheConfig:
    block_size: int = 64
    num_blocks: int | None = None
    # Fraction of free device memory the KV pool may take when num_blocks is None.
    memory_fraction: float = 0.5
    # Reuse the KV blocks of a shared prompt prefix (full-attention models only).
    enable_prefix_caching: bool = False


@dataclass
class EngineConfig:
    model_config: ModelConfig
    parallel_config: ParallelConfig = field(default_factory=ParallelConfig)
    compilation_config: CompilationConfig = field(default_factory=CompilationConfig)
    cache_config: CacheConfig = field(default_factory=CacheConfig)
    additional_config: dict[str, Any] = field(default_factory=dict)
    max_num_seqs: int = 256
    # Prompt tokens one prefill step may compute (chunked prefill); None = whole prompts.
    max_num_batched_tokens: int | None = None
    # Launch decode step t+1 before reading step t's tokens back (decode steps
    # without penalties / logprobs / min_tokens and with no request waiting);
    # a step() then returns the previous step's tokens.
    async_scheduling: bool = False


__all__ = ["CacheConfig", "CompilationConfig", "EngineConfig", "ModelConfig", "ParallelConfig"]
