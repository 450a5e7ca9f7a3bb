"""Prefix caching: refcounted blocks, chained block hashes, reuse, eviction, reset (CPU, fp32)."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import CacheConfig, EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.kv_cache import BlockAllocator, block_hashes


def test_allocator_refcounts_cache_and_eviction():
    a = BlockAllocator(5)  # blocks 1..4 usable
    x = a.allocate(2)
    hs = block_hashes(list(range(8)), 4)
    for b, h in zip(x, hs):
        a.register(b, h)
    assert a.lookup(hs) == x  # shared while still in use
    a.free(x)
    a.free(x)  # both users gone: cached, evictable, still counted free
    assert a.num_free == 4 and a.num_cached == 2
    y = a.allocate(2)  # empty blocks first
    assert not set(y) & set(x) and a.num_cached == 2
    z = a.allocate(1)  # then the least recently released cached block
    assert z[0] == x[1] or z[0] == x[0]
    assert a.num_cached == 1
    a.free(y + z)
    assert a.reset_cache() == 1 and a.num_cached == 0 and a.num_free == 4
    assert a.lookup(hs) == [] and a.hits == 2 and a.queries == 3  # a lookup stops at its first miss
    with pytest.raises(MemoryError):
        a.allocate(5)


def test_block_hashes_chain():
    h1 = block_hashes([1, 2, 3, 4, 5, 6, 7, 8, 9], 4)
    assert len(h1) == 2
    h2 = block_hashes([0, 2, 3, 4, 5, 6, 7, 8], 4)
    assert h1[1] != h2[1]  # a different first block changes every later hash


def _engine(preset="tiny-dsv2", cache=True, num_blocks=None, block_size=4):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96),
                      cache_config=CacheConfig(block_size=block_size, num_blocks=num_blocks,
                                               enable_prefix_caching=cache), max_num_seqs=4)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))


def _prefill_lens(eng):
    seen = []
    orig = eng.runner.prefill

    def spy(tokens, tables, starts, slots=None, **kw):
        seen.append([(len(t), s) for t, s in zip(tokens, starts)])
        return orig(tokens, tables, starts, slots, **kw)

    eng.runner.prefill = spy
    return seen


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3-moe", "tiny-dsv32"])
def test_shared_prefix_is_reused_and_outputs_do_not_change(preset):
    shared = list(range(100, 120))  # five blocks of four
    a, b = shared + [7, 8, 9], shared + [3, 1]
    want = _engine(preset, cache=False).generate([a], 5) + _engine(preset, cache=False).generate([b], 5)
    eng = _engine(preset)
    seen = _prefill_lens(eng)
    got = eng.generate([a], 5) + eng.generate([b], 5)
    assert got == want
    # the second prompt computed only what follows the five cached blocks
    assert seen == [[(23, 0)], [(2, 20)]]
    assert eng.kv.allocator.hits == 5
    # a whole cached prompt still computes its last token
    seen.clear()
    assert eng.generate([a], 5) == want[:1]
    assert seen == [[(3, 20)]]


def test_eviction_under_pressure_keeps_outputs_right():
    eng = _engine(num_blocks=12)
    prompts = [[i] * 9 + [i + 1] for i in range(1, 6)]
    want = [_engine(cache=False).generate([p], 3)[0] for p in prompts]
    for p, w in zip(prompts, want):
        assert eng.generate([p], 3)[0] == w
    assert eng.generate([prompts[-1]], 3)[0] == want[-1]
    assert eng.reset_prefix_cache() > 0 and eng.kv.allocator.num_cached == 0


def test_hybrid_models_do_not_share_blocks():
    assert _engine("tiny-qwen3.5").prefix_caching is False
    assert _engine("tiny-dsv2").prefix_caching is True
    assert _engine("tiny-dsv2", cache=False).prefix_caching is False


def test_server_reports_and_resets_the_prefix_cache():
    import threading
    import time

    import requests
    import uvicorn

    from afd_plugin_b200.runtime.launcher import free_port
    from afd_plugin_b200.serving import EngineLoop, build_app

    loop = EngineLoop(_engine()).start()
    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(loop), host="127.0.0.1", port=port, log_level="warning"))
    threading.Thread(target=srv.run, daemon=True).start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if requests.get(url + "/health", timeout=2).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    try:
        p = list(range(200, 217))
        for _ in range(2):
            requests.post(url + "/v1/completions", json={"prompt": p, "max_tokens": 2}, timeout=60)
        m = requests.get(url + "/metrics", timeout=5).json()
        assert m["prefix_cache_hit_rate"] == 0.8  # the first lookup stops at its miss, the second hits 4 blocks
        r = requests.post(url + "/reset_prefix_cache", timeout=10).json()
        assert r["reset"] is True and r["cached_blocks_dropped"] == 4
    finally:
        srv.should_exit = True
        loop.stop()
