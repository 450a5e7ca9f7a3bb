"""Prefill -> decode hand-off between two engines (CPU, fp32).

A prefill engine runs the prompt with ``hold_kv``; its cache rows (MLA
latents, GQA K/V, Gated DeltaNet conv + delta-rule state) move to a second
engine as a payload, which decodes the rest.  The tokens must equal one
engine generating everything.
"""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime import kv_transfer as kt
from afd_plugin_b200.runtime.engine import LLMEngine


def _engine(preset: str, seed: int = 0, max_num_seqs: int = 4) -> LLMEngine:
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96),
                      max_num_seqs=max_num_seqs)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=seed, max_positions=96))


def _prompts(vocab: int, n: int = 3):
    g = torch.Generator().manual_seed(4)
    return [torch.randint(0, vocab, (5 + 3 * i,), generator=g).tolist() for i in range(n)]


def _drain(eng: LLMEngine) -> None:
    while eng.has_unfinished():
        eng.step()


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3-moe", "tiny-qwen3.5"])
@pytest.mark.parametrize("prefill_tokens", [1, 3])
def test_handoff_matches_single_engine(preset, prefill_tokens):
    max_tokens = 6
    ref_eng = _engine(preset)
    prompts = _prompts(ref_eng.model.arch.vocab_size)
    ref = ref_eng.generate(prompts, max_tokens)

    pre, dec = _engine(preset), _engine(preset)
    rids = [pre.add_request(p, prefill_tokens, hold_kv=True) for p in prompts]
    _drain(pre)
    assert set(pre.held) == set(rids)
    free_before = pre.kv.allocator.num_free
    blobs = [pre.export_kv(r) for r in rids]
    assert not pre.held and pre.kv.allocator.num_free > free_before

    ids = []
    for p, blob in zip(prompts, blobs):
        rid, tokens = dec.add_prefilled_request(blob, max_tokens - prefill_tokens + 1)
        assert tokens[: len(p)] == p
        ids.append(rid)
    _drain(dec)
    for i, (p, rid) in enumerate(zip(prompts, ids)):
        got = pre.finished[rids[i]].output[:-1] + dec.finished[rid].output
        assert got == ref[i], (preset, i)


def test_held_requests_expire_and_release():
    eng = _engine("tiny-dsv2")
    total = eng.kv.allocator.num_free
    rid = eng.add_request([1, 2, 3], 1, hold_kv=True)
    _drain(eng)
    assert eng.kv.allocator.num_free < total
    assert eng.expire_held(3600.0) == []
    assert eng.expire_held(-1.0) == [rid]
    assert eng.kv.allocator.num_free == total
    assert eng.release_kv(rid) is False
    with pytest.raises(KeyError):
        eng.export_kv(rid)


def test_payload_rejected_by_other_model():
    pre = _engine("tiny-dsv2")
    rid = pre.add_request([5, 6, 7, 8], 1, hold_kv=True)
    _drain(pre)
    blob = pre.export_kv(rid)
    other = _engine("tiny-qwen3-moe")
    with pytest.raises(ValueError, match="no cache for"):
        other.add_prefilled_request(blob, 4)
    with pytest.raises(ValueError):
        kt.unpack(b"garbage!")


def test_imported_requests_wait_for_a_batch_slot():
    pre = _engine("tiny-dsv2", max_num_seqs=4)
    prompts = _prompts(pre.model.arch.vocab_size, n=3)
    rids = [pre.add_request(p, 1, hold_kv=True) for p in prompts]
    _drain(pre)
    dec = _engine("tiny-dsv2", max_num_seqs=1)
    ids = [dec.add_prefilled_request(pre.export_kv(r), 3)[0] for r in rids]
    dec.step()
    assert len(dec.running) == 1 and len(dec._kv_waiting) == 2
    _drain(dec)
    assert all(len(dec.finished[i].output) == 3 for i in ids)
    # one transferred token and nothing else: finishes without a model step
    pre2 = _engine("tiny-dsv2")
    r = pre2.add_request(prompts[0], 1, hold_kv=True)
    _drain(pre2)
    rid, _ = dec.add_prefilled_request(pre2.export_kv(r), 1)
    assert dec.step() == {}
    assert dec.finished[rid].output == pre2.finished[r].output


def test_imported_requests_wait_for_free_blocks():
    from afd_plugin_b200.engine_config import CacheConfig

    arch = get_preset("tiny-dsv2")
    pre = _engine("tiny-dsv2")
    prompts = _prompts(arch.vocab_size)
    blobs = []
    for p in prompts:
        rid = pre.add_request(p, 1, hold_kv=True)
        _drain(pre)
        blobs.append(pre.export_kv(rid))
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96),
                      cache_config=CacheConfig(block_size=4, num_blocks=9), max_num_seqs=4)
    dec = LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))
    ids = [dec.add_prefilled_request(b, 3)[0] for b in blobs]
    _drain(dec)  # no MemoryError: imports wait for blocks
    ref = _engine("tiny-dsv2").generate(prompts, 3)
    assert [dec.finished[i].output for i in ids] == ref
