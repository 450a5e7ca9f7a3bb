"""Async scheduling: decode step t+1 launches before step t's tokens are read; outputs equal the sync engine's."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import CacheConfig, EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.sampling import SamplingParams


def _engine(async_scheduling: bool, block_size: int = 4, num_blocks: int | None = None,
            preset: str = "tiny-dsv2") -> LLMEngine:
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96),
                      cache_config=CacheConfig(block_size=block_size, num_blocks=num_blocks), max_num_seqs=8,
                      async_scheduling=async_scheduling)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))


PROMPTS = [[3, 9, 4], [7, 1, 2, 8, 5, 6], [11, 12], [5, 5, 5, 5], [2, 30, 17, 9, 1]]
MAX_TOKENS = [9, 4, 13, 7, 11]


def _run(eng: LLMEngine, stop: dict[int, int] | None = None) -> tuple[list[list[int]], int]:
    ids = []
    for i, (p, m) in enumerate(zip(PROMPTS, MAX_TOKENS)):
        sp = SamplingParams(stop_token_ids=[stop[i]]) if stop and i in stop else None
        ids.append(eng.add_request(p, m, sampling=sp))
    while eng.has_unfinished():
        eng.step()
    return [eng.finished[i].output for i in ids], eng.num_async_steps


def test_async_equals_sync_with_lengths_and_stop_tokens():
    ref, _ = _run(_engine(False))
    # stop request 0 at its 4th token and request 3 at its 2nd: rows end between steps both ways
    stop = {0: ref[0][3], 3: ref[3][1]}
    want, _ = _run(_engine(False), stop)
    got, pipelined = _run(_engine(True), stop)
    assert got == want
    assert pipelined > 5  # most decode steps launched ahead of their predecessor's read-back
    assert len(want[0]) <= 4 and len(want[3]) <= 2


def test_async_step_returns_previous_tokens_and_drains_for_new_work():
    eng = _engine(True)
    a = eng.add_request(PROMPTS[0], 12)
    first = eng.step()  # prefill: synchronous, returns the first token
    assert list(first) == [a]
    assert eng.step() == {}  # the first pipelined decode launches; nothing read back yet
    got = eng.step()  # launches the next step and returns the previous one's token
    assert list(got) == [a] and eng._inflight is not None
    b = eng.add_request(PROMPTS[1], 5)
    drained = eng.step()  # a prompt is waiting: read the step in flight, launch nothing
    assert list(drained) == [a] and eng._inflight is None
    while eng.has_unfinished():
        eng.step()
    ref = _engine(False)
    ra = ref.add_request(PROMPTS[0], 12)
    rb = ref.add_request(PROMPTS[1], 5)
    while ref.has_unfinished():
        ref.step()
    assert eng.finished[a].output == ref.finished[ra].output
    assert eng.finished[b].output == ref.finished[rb].output


def test_async_abort_drops_the_token_in_flight():
    eng = _engine(True)
    ids = [eng.add_request(p, m) for p, m in zip(PROMPTS[:3], (10, 10, 10))]
    eng.step()
    for _ in range(3):
        eng.step()
    n = len(eng.running[1].output)
    assert eng.abort(ids[1])
    while eng.has_unfinished():
        eng.step()
    assert len(eng.finished[ids[1]].output) == n and eng.finished[ids[1]].aborted
    assert all(len(eng.finished[i].output) == 10 for i in (ids[0], ids[2]))
    assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks - 1  # every block back (block 0 pads)


def test_async_falls_back_when_blocks_run_short():
    """With too few free KV blocks for the next positions, the engine drains and the sync path preempts."""
    ref, eng = _engine(False, block_size=2, num_blocks=16), _engine(True, block_size=2, num_blocks=16)
    want, _ = _run(ref)
    got, pipelined = _run(eng)
    assert got == want
    assert ref.num_preemptions > 0 and eng.num_preemptions > 0 and pipelined > 0


def test_async_reads_the_device_status_behind_each_step():
    """An executor with a device status word: the async engine copies the word behind every step and
    checks the copy after the step's event (no blocking read of the live word), and a set word raises."""
    from afd_plugin_b200.runtime.ffn_executor import LocalFFNExecutor

    class Watched(LocalFFNExecutor):
        def __init__(self, model):
            super().__init__(model)
            self.word = torch.zeros(1, dtype=torch.int32)
            self.seen = []

        def device_status_word(self):
            return self.word

        def check_device_status(self, status=None):
            assert status is not None  # the engine passes the copy it read behind the step
            self.seen.append(status)
            if status:
                raise RuntimeError(f"status {status}")

    eng = _engine(True)
    eng.ffn = eng.runner.ffn = Watched(eng.model)
    eng.add_request(PROMPTS[0], 12)
    eng.step()  # prefill (sync path: the executor's own check runs with no argument only there)
    eng.ffn.seen.clear()
    for _ in range(3):
        eng.step()
    assert eng.ffn.seen == [0, 0] and eng.num_async_steps == 3
    eng.ffn.word[0] = 7  # a bounded wait expired during the next launched step
    eng.step()  # reads the step launched before the word was set: still clean
    with pytest.raises(RuntimeError, match="status 7"):
        eng.step()


def _engine_with(async_scheduling: bool, **cfg) -> LLMEngine:
    arch = get_preset("tiny-dsv2")
    cache = CacheConfig(block_size=4, enable_prefix_caching=cfg.pop("prefix", False))
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96),
                      cache_config=cache, max_num_seqs=8, async_scheduling=async_scheduling, **cfg)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))


@pytest.mark.parametrize("cfg", [{"max_num_batched_tokens": 5}, {"prefix": True}], ids=["chunked", "prefix"])
def test_async_with_staggered_arrivals(cfg):
    """Requests arrive while others decode (chunked prefill or prefix-cache hits in between): every
    request's tokens equal the sync engine's under the same arrival schedule (arrivals keyed to the
    number of tokens the first request has produced)."""
    shared = [8, 8, 1, 2, 3, 4, 5, 6]  # two full 4-token blocks shared by the later prompts
    arrivals = {0: [shared + [9]], 3: [shared + [7, 7], [4, 5]], 6: [shared + [1]]}

    def run(async_scheduling):
        eng = _engine_with(async_scheduling, **dict(cfg))
        first = eng.add_request(PROMPTS[1], 14)
        ids, done = [first], set()
        while eng.has_unfinished():
            n = len(eng.request(first).output) if first not in eng.finished else 99
            for at, prompts in arrivals.items():
                if n >= at and at not in done:
                    done.add(at)
                    ids += [eng.add_request(p, 8) for p in prompts]
            eng.step()
        return [eng.finished[i].output for i in ids], eng.num_async_steps

    want, _ = run(False)
    got, n_async = run(True)
    assert got == want and n_async > 0


def test_async_sampled_requests_match_sync():
    """Seeded temperature / top-k / top-p requests (each its own generator) pipelined: tokens equal the
    sync engine's; a penalised request drains and runs synchronously."""
    sps = [SamplingParams(temperature=0.8, seed=11), SamplingParams(temperature=1.2, top_k=20, seed=5),
           SamplingParams(temperature=0.7, top_p=0.9, seed=3), SamplingParams()]

    def run(async_scheduling, extra=None):
        eng = _engine(async_scheduling)
        ids = [eng.add_request(p, m, sampling=sp) for p, m, sp in zip(PROMPTS, MAX_TOKENS, sps)]
        if extra is not None:
            ids.append(eng.add_request(PROMPTS[4], 6, sampling=extra))
        while eng.has_unfinished():
            eng.step()
        return [eng.finished[i].output for i in ids], eng.num_async_steps

    want, _ = run(False)
    got, n_async = run(True)
    assert got == want and n_async >= 8
    pen = SamplingParams(temperature=0.9, seed=2, presence_penalty=0.5)
    want, _ = run(False, pen)
    got, n_async = run(True, pen)
    assert got == want and n_async >= 4  # pipelined again once the penalised request ends


@pytest.mark.parametrize("preset", ["tiny-qwen3-moe", "tiny-qwen3.5", "tiny-dsv4", "tiny-dsv1", "tiny-dsv32"])
def test_async_equals_sync_across_model_families(preset):
    """GQA + QK-norm, Gated DeltaNet state rows, mHC streams with hash routing (the router reads the
    device-gathered input ids), DeepSeek V1, and DeepSeek sparse attention (contexts cross index_topk
    while steps are in flight: the sparse decision counts the token in flight): pipelined tokens equal
    the sync engine's."""
    want, _ = _run(_engine(False, preset=preset))
    got, n_async = _run(_engine(True, preset=preset))
    assert got == want and n_async >= 8


@pytest.mark.parametrize("async_scheduling", [False, True], ids=["sync", "async"])
def test_sparse_attention_decision_counts_the_token_in_flight(async_scheduling):
    """DeepSeek sparse attention selects positions exactly on the steps whose longest context exceeds
    index_topk; with a step in flight the staged context is one token longer than the host's view."""
    eng = _engine(async_scheduling, preset="tiny-dsv32")
    topk = eng.model.arch.index_topk
    seen = []
    inner = eng.runner.decode_step

    def spy(batch, **kw):
        seen.append((bool(eng.runner.sparse_decode), int(eng._n_lens[:batch].max())))
        return inner(batch, **kw)

    eng.runner.decode_step = spy
    for p, m in zip(PROMPTS, MAX_TOKENS):
        eng.add_request(p, m)
    while eng.has_unfinished():
        eng.step()
    assert any(s for s, _ in seen) and not all(s for s, _ in seen)
    assert all(s == (longest > topk) for s, longest in seen)


def test_close_reads_back_the_step_in_flight():
    eng = _engine(True)
    rid = eng.add_request(PROMPTS[0], 12)
    for _ in range(4):
        eng.step()
    assert eng._inflight is not None
    n = len(eng.request(rid).output)
    eng.close()
    assert eng._inflight is None and len(eng.request(rid).output) == n + 1
