"""Attention tensor parallelism on CPU: head shards sum to the unsharded layer; gloo AFD parity."""

from dataclasses import dataclass

import pytest
import torch

from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.models.layers import AttentionMetadata, TPInfo
from afd_plugin_b200.runtime.kv_cache import KVCache


@dataclass(frozen=True)
class _NoReduce(TPInfo):
    """Shard without summing: the test adds the partial outputs itself."""

    def all_reduce(self, x):
        return x


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-dsv3", "tiny-qwen3-moe"])
def test_head_shards_sum_to_full_attention(preset):
    arch = get_preset(preset)
    torch.manual_seed(0)
    full = build_model(arch, role="attention", dtype=torch.float32, seed=3)
    shards = [build_model(arch, role="attention", dtype=torch.float32, seed=3, tp=_NoReduce(r, 2, None))
              for r in range(2)]
    T = 5
    h = torch.randn(T, arch.hidden_size) * 0.5
    meta = AttentionMetadata(positions=torch.arange(T), slot_mapping=torch.arange(T),
                             block_table=torch.zeros(1, 2, dtype=torch.int32), seq_lens=torch.tensor([T]),
                             is_decode=False, prefill_seqs=[(0, T, 0)])

    def run(m):
        kv = KVCache(m.cache_arch, 4, 64, torch.float32, "cpu")
        return m.layers[0].self_attn(m.layers[0].input_layernorm(h), meta, kv.layer(0), m.cos_sin)

    want = run(full)
    got = run(shards[0]) + run(shards[1])
    torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
    assert shards[0].layers[0].self_attn.o_proj.shape[1] * 2 == full.layers[0].self_attn.o_proj.shape[1]


def test_tp_requires_divisible_heads():
    arch = get_preset("tiny-qwen3-moe")  # 4 query heads, 2 KV heads
    with pytest.raises(ValueError):
        build_model(arch, role="attention", dtype=torch.float32, tp=_NoReduce(0, 3, None))
