"""Debug-mode index validation in front of the kernels (AFD_DEBUG_CHECKS)."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200 import ops
from afd_plugin_b200.ops import checks
from afd_plugin_b200.ops.checks import KernelInputError


@pytest.fixture
def debug_checks():
    was = checks.enabled()
    checks.enable(True)
    yield
    checks.enable(was)


def _mla_inputs(nb=4, bs=8, B=2, H=2, D=16):
    q = torch.randn(B, H, D)
    kv = torch.randn(nb, bs, D)
    table = torch.tensor([[1, 2, 0], [3, 0, 0]], dtype=torch.int32)
    lens = torch.tensor([12, 5], dtype=torch.int32)
    return q, kv, table, lens


def test_valid_inputs_pass_and_unused_entries_are_ignored(debug_checks):
    q, kv, table, lens = _mla_inputs()
    table[1, 2] = 12345  # beyond sequence 1's blocks: never read
    out = ops.mla_decode(q, kv, table, lens, 0.1, 12)
    assert out.shape == (2, 2, 12)


def test_block_outside_pool_is_reported(debug_checks):
    q, kv, table, lens = _mla_inputs()
    table[0, 1] = 4
    with pytest.raises(KernelInputError, match=r"block_table\[0, 1\] = 4 outside \[0, 4\)"):
        ops.mla_decode(q, kv, table, lens, 0.1, 12)
    table[0, 1] = -1
    with pytest.raises(KernelInputError, match="block_table"):
        ops.gqa_decode(torch.randn(2, 4, 8), torch.randn(4, 8, 2, 8), torch.randn(4, 8, 2, 8), table, lens, 0.1)


def test_sequence_longer_than_its_table(debug_checks):
    q, kv, table, lens = _mla_inputs()
    lens[1] = 25
    with pytest.raises(KernelInputError, match=r"seq_lens\[1\] = 25"):
        ops.mla_decode(q, kv, table, lens, 0.1, 12)
    lens[1] = 0
    with pytest.raises(KernelInputError, match=r"seq_lens\[1\] = 0"):
        ops.mla_decode(q, kv, table, lens, 0.1, 12)


def test_cache_slots_checked(debug_checks):
    kc, vc = torch.zeros(4, 8, 2, 8), torch.zeros(4, 8, 2, 8)
    k = v = torch.randn(3, 2, 8)
    ops.gqa_cache_write(kc, vc, k, v, torch.tensor([0, 9, 31]))
    with pytest.raises(KernelInputError, match=r"slot_mapping\[2\] = 32 outside \[0, 32\)"):
        ops.gqa_cache_write(kc, vc, k, v, torch.tensor([0, 9, 32]))


def test_expert_ids_and_weights_checked(debug_checks):
    x = torch.randn(3, 8)
    w13, w2 = torch.randn(4, 2 * 6, 8), torch.randn(4, 8, 6)
    ids = torch.tensor([[0, 1], [2, 3], [1, 2]])
    wts = torch.full((3, 2), 0.5)
    ops.moe_experts(x, w13, w2, wts, ids)
    with pytest.raises(KernelInputError, match="expert id"):
        ops.moe_experts(x, w13, w2, wts, ids - 1)
    wts[1, 0] = float("nan")
    with pytest.raises(KernelInputError, match="routing weight"):
        ops.moe_experts(x, w13, w2, wts, ids)
    with pytest.raises(KernelInputError, match=r"outside \[0, 4\)"):
        ops.topk_route(torch.randn(3, 4), 2, forced_ids=torch.tensor([[0, 4], [1, 2], [3, 0]]))
    with pytest.raises(KernelInputError, match="state slot"):
        checks.state_slots("gdn", torch.tensor([0, 5]), max_seqs=5)


def test_checks_off_by_default_cost_nothing():
    assert checks.ENV == "AFD_DEBUG_CHECKS"
    was = checks.enabled()
    checks.enable(False)
    try:
        checks.paged_attention("x", torch.tensor([[99]]), torch.tensor([100]), num_blocks=1, block_size=1)
    finally:
        checks.enable(was)


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3-moe", "tiny-qwen3.5"])
def test_engine_runs_clean_under_checks(debug_checks, preset):
    from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
    from afd_plugin_b200.models import build_model, get_preset
    from afd_plugin_b200.runtime.engine import LLMEngine

    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64), max_num_seqs=3)
    eng = LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64))
    out = eng.generate([[1, 2, 3], [4, 5, 6, 7, 8, 9, 10, 11, 12], [7]], 5)
    assert all(len(o) == 5 for o in out)
