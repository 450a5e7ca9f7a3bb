"""Decode-step input staging: vectorised rows and cached block-table rows equal a per-request rebuild."""

from __future__ import annotations

import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.kv_cache import PAD_BLOCK


def _engine(max_num_seqs=6, block_size=4):
    from afd_plugin_b200.engine_config import CacheConfig

    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64),
                      cache_config=CacheConfig(block_size=block_size), max_num_seqs=max_num_seqs)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64))


def _expected(eng, reqs, run_b):
    bs = eng.block_size
    rows = []
    for r in reqs:
        p = r.num_tokens - 1
        table = list(r.blocks) + [PAD_BLOCK] * (eng.max_blocks_per_seq - len(r.blocks))
        rows.append((r.output[-1], p, r.blocks[p // bs] * bs + p % bs, p + 1, r.state_slot, table))
    for _ in range(len(reqs), run_b):
        rows.append((0, 0, PAD_BLOCK * bs, 1, eng.runner.pad_state_slot, [PAD_BLOCK] * eng.max_blocks_per_seq))
    return rows


def _staged(eng, run_b):
    return [(int(eng._n_ids[i]), int(eng._n_pos[i]), int(eng._n_slot[i]), int(eng._n_lens[i]),
             int(eng._n_state[i]), eng._n_table[i].tolist()) for i in range(run_b)]


def test_staging_tracks_block_growth_and_batch_changes():
    eng = _engine()
    for n, mt in ((3, 9), (6, 2), (5, 12), (2, 5)):
        eng.add_request(list(range(1, n + 1)), mt)
    eng.step()  # prefill
    seen_growth = False
    while eng.running:
        reqs = list(eng.running)
        blocks_before = {r.req_id: len(r.blocks) for r in reqs}
        run_b = len(reqs) + 2  # two padding rows, as a padded graph batch would add
        eng._stage_decode_inputs(reqs, run_b)
        seen_growth |= any(len(r.blocks) > blocks_before[r.req_id] for r in reqs)
        assert _staged(eng, run_b) == _expected(eng, reqs, run_b)
        eng.step()  # requests finish at different steps: rows shift between steps
    assert seen_growth
    # a shorter batch after a longer one re-pads the rows it no longer uses
    eng.add_request([7, 8], 3)
    eng.step()
    eng._stage_decode_inputs(eng.running, 4)
    assert _staged(eng, 4) == _expected(eng, eng.running, 4)


def test_staging_a_full_batch_is_cheap():
    """Host prep of a 256-request decode step stays far below a device step (about 10 ms on B200)."""
    import statistics
    import time

    from afd_plugin_b200.runtime.engine import Request

    from afd_plugin_b200.engine_config import CacheConfig

    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=1344),
                      cache_config=CacheConfig(block_size=64, num_blocks=200), max_num_seqs=256)
    eng = LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64))
    reqs = []
    for i in range(256):
        r = Request(i, [1] * 1024, 256)
        r.output = [5] * 40
        r.blocks = list(range(1 + 17 * (i % 8), 1 + 17 * (i % 8) + 17))
        r.state_slot = 0
        reqs.append(r)
    eng._stage_decode_inputs(reqs, 256)  # first pass writes every block-table row
    times = []
    for _ in range(20):
        t0 = time.perf_counter()
        eng._stage_decode_inputs(reqs, 256)
        times.append(time.perf_counter() - t0)
    assert statistics.median(times) < 2e-3
