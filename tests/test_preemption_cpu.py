"""KV-cache pressure: admission waits for blocks, running requests are preempted and recomputed (CPU, fp32)."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import CacheConfig, EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine


def _engine(preset, num_blocks=None, prefix=False, budget=None):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64),
                      cache_config=CacheConfig(block_size=4, num_blocks=num_blocks, enable_prefix_caching=prefix),
                      max_num_seqs=4, max_num_batched_tokens=budget)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64))


def _prompts(vocab):
    g = torch.Generator().manual_seed(11)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in (9, 14, 6, 11)]


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3-moe", "tiny-qwen3.5", "tiny-dsv32"])
def test_tight_cache_preempts_and_outputs_do_not_change(preset):
    prompts = _prompts(get_preset(preset).vocab_size)
    want = _engine(preset).generate(prompts, 10)
    eng = _engine(preset, num_blocks=13)  # 12 usable blocks: four requests need up to 6 each
    assert eng.generate(prompts, 10) == want
    assert eng.num_preemptions > 0
    assert eng.kv.allocator.num_free == 12


def test_preemption_with_prefix_cache_and_chunks():
    prompts = _prompts(1024)
    want = _engine("tiny-dsv2").generate(prompts, 10)
    eng = _engine("tiny-dsv2", num_blocks=13, prefix=True, budget=6)
    assert eng.generate(prompts, 10) == want
    assert eng.num_preemptions > 0


def test_request_larger_than_the_cache_is_refused():
    eng = _engine("tiny-dsv2", num_blocks=5)
    with pytest.raises(ValueError, match="more KV blocks than the cache holds"):
        eng.add_request(list(range(10)), 10)
