"""Chunked prefill: prompts computed over several steps within a token budget (CPU, fp32)."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import CacheConfig, EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine


def _engine(preset, budget=None, prefix=False):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96),
                      cache_config=CacheConfig(block_size=4, enable_prefix_caching=prefix), max_num_seqs=4,
                      max_num_batched_tokens=budget)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))


def _prompts(vocab):
    g = torch.Generator().manual_seed(8)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in (23, 6, 17)]


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3-moe", "tiny-qwen3.5", "tiny-dsv32", "tiny-dsv4"])
def test_chunked_outputs_equal_whole_prompt_prefill(preset):
    vocab = get_preset(preset).vocab_size
    prompts = _prompts(vocab)
    want = _engine(preset).generate(prompts, 5)
    eng = _engine(preset, budget=7)
    chunks = []
    orig = eng.runner.prefill

    def spy(tokens, tables, starts, slots=None, **kw):
        chunks.append(sum(len(t) for t in tokens))
        return orig(tokens, tables, starts, slots, **kw)

    eng.runner.prefill = spy
    assert eng.generate(prompts, 5) == want
    assert max(chunks) <= 7 and sum(chunks) == sum(len(p) for p in prompts)


def test_running_requests_keep_decoding_while_a_long_prompt_chunks():
    eng = _engine("tiny-dsv2", budget=4)
    short = eng.add_request([1, 2, 3], 8)
    eng.step()  # the short prompt fits one chunk
    long_id = eng.add_request(list(range(10, 40)), 2)
    phases = []
    while not eng.request(long_id).output:
        eng.step()
        phases.append(eng._last_phase)
    # prefill chunks alternate with decode steps of the running request
    assert phases.count("prefill") == 8 and "decode" in phases
    # while the short request runs, no two prefill chunks come back to back
    running_until = len(eng.request(short).output) - 1  # decode steps the short request took
    assert running_until >= 1
    assert not any(a == b == "prefill" for a, b in zip(phases[: 2 * running_until], phases[1 : 2 * running_until]))


def test_chunked_prefill_with_prefix_cache_and_abort():
    prompts = _prompts(1024)
    want = _engine("tiny-dsv2").generate([prompts[0]], 4)[0]
    eng = _engine("tiny-dsv2", budget=5, prefix=True)
    assert eng.generate([prompts[0]], 4)[0] == want
    assert eng.generate([prompts[0]], 4)[0] == want  # second time: cached blocks, fewer chunks
    rid = eng.add_request(list(range(50, 80)), 4)
    eng.step()
    assert eng.request(rid) in eng.prefilling
    assert eng.abort(rid) and eng.finished[rid].aborted and not eng.prefilling
    while eng.has_unfinished():
        eng.step()
