"""DeepSeek sparse attention (DeepSeek-V3.2 / GLM-MoE-DSA lightning indexer) on CPU, fp32."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.ops import reference as ref
from afd_plugin_b200.runtime.engine import LLMEngine


def _engine(arch, max_len=128, max_num_seqs=4):
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=max_len),
                      max_num_seqs=max_num_seqs)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=max_len))


def _prompts(vocab, lens, seed=5):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


def test_index_scores_and_selection_match_a_loop():
    g = torch.Generator().manual_seed(0)
    q, w, k = torch.randn(3, 4, 8, generator=g), torch.randn(3, 4, generator=g), torch.randn(10, 8, generator=g)
    s = ref.dsa_index_scores(q, w, k)
    for t in range(3):
        for n in range(10):
            want = sum(float(w[t, h]) * max(0.0, float(q[t, h] @ k[n])) for h in range(4))
            assert abs(float(s[t, n]) - want) < 1e-4
    valid = torch.arange(10)[None, :] <= torch.tensor([1, 5, 9])[:, None]
    pos = ref.dsa_select(s, valid, 4)
    assert pos.shape == (3, 4)
    assert sorted(p for p in pos[0].tolist() if p >= 0) == [0, 1] and (pos[0] < 0).sum() == 2
    for t, last in enumerate((1, 5, 9)):
        kept = [p for p in pos[t].tolist() if p >= 0]
        assert all(p <= last for p in kept)
        best = s[t, : last + 1].topk(min(4, last + 1)).indices.tolist()
        assert sorted(kept) == sorted(best)


def test_config_parsing_and_cache_geometry():
    hf = {"architectures": ["DeepseekV32ForCausalLM"], "model_type": "deepseek_v32", "hidden_size": 64,
          "num_hidden_layers": 2, "vocab_size": 100, "num_attention_heads": 2, "q_lora_rank": 32,
          "kv_lora_rank": 16, "qk_nope_head_dim": 8, "qk_rope_head_dim": 8, "v_head_dim": 8,
          "intermediate_size": 64, "index_topk": 2048, "index_n_heads": 64, "index_head_dim": 128}
    a = ModelArchConfig.from_hf_config(hf)
    assert a.has_indexer and (a.index_topk, a.index_n_heads, a.index_head_dim) == (2048, 64, 128)
    assert a.kv_cache_width == 16 + 8 + 128
    eng = _engine(get_preset("tiny-dsv32"))
    assert eng.kv.index_k.shape[-1] == 48 and isinstance(eng.kv.layer(0), tuple)


def test_short_sequences_match_dense_attention():
    """Within index_topk every position is selected: outputs equal the dense model's."""
    sparse_arch = get_preset("tiny-dsv32")
    dense_arch = sparse_arch.scaled(index_topk=0)
    prompts = _prompts(sparse_arch.vocab_size, (3, 5, 4))
    out_sparse = _engine(sparse_arch).generate(prompts, 3)  # longest sequence: 5 + 3 - 1 = 7 < 8
    out_dense = _engine(dense_arch).generate(prompts, 3)
    assert out_sparse == out_dense


def test_long_sequences_are_sparse_and_decode_matches_recompute():
    """Past index_topk the selection changes the output, and a decode step equals a fresh prefill."""
    arch = get_preset("tiny-dsv32")
    prompts = _prompts(arch.vocab_size, (20, 13, 30))
    eng = _engine(arch)
    outs = eng.generate(prompts, 5)
    dense = _engine(arch.scaled(index_topk=0)).generate(prompts, 5)
    assert outs != dense
    for p, o in zip(prompts, outs):
        for i in range(1, len(o)):
            fresh = _engine(arch)
            assert fresh.generate([p + o[:i]], 1)[0][0] == o[i]


@pytest.mark.parametrize("prefill_tokens", [1, 4])
def test_kv_handoff_carries_indexer_keys(prefill_tokens):
    arch = get_preset("tiny-dsv32")
    prompts = _prompts(arch.vocab_size, (12, 20))
    ref_out = _engine(arch).generate(prompts, 6)
    pre, dec = _engine(arch), _engine(arch)
    rids = [pre.add_request(p, prefill_tokens, hold_kv=True) for p in prompts]
    while pre.has_unfinished():
        pre.step()
    got = []
    for p, rid in zip(prompts, rids):
        new, _ = dec.add_prefilled_request(pre.export_kv(rid), 6 - prefill_tokens + 1)
        while dec.has_unfinished():
            dec.step()
        got.append(pre.finished[rid].output[:-1] + dec.finished[new].output)
    assert got == ref_out


def test_indexer_weights_are_attention_role_and_load_by_name():
    from afd_plugin_b200.models import weight_roles

    arch = get_preset("tiny-dsv32")
    name = "model.layers.1.self_attn.indexer.wq_b.weight"
    assert weight_roles(name, arch, compute_gate_on_attention=False) == {"attention"}
    ffn = build_model(arch, role="ffn", dtype=torch.float32, seed=0)
    assert all("indexer" not in s.name for s in ffn.param_specs())


def test_sparse_kernel_selection_by_head_count(monkeypatch):
    """The gather kernel is the default up to 32 heads; the switch forces either path."""
    from afd_plugin_b200 import ops

    monkeypatch.delenv("AFD_SPARSE_MLA_KERNEL", raising=False)
    assert ops.sparse_kernel_enabled(16) and ops.sparse_kernel_enabled(32)
    assert not ops.sparse_kernel_enabled(128)
    monkeypatch.setenv("AFD_SPARSE_MLA_KERNEL", "1")
    assert ops.sparse_kernel_enabled(128)
    monkeypatch.setenv("AFD_SPARSE_MLA_KERNEL", "0")
    assert not ops.sparse_kernel_enabled(16)
