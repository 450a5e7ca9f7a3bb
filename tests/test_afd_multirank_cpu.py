"""AFD over real processes (gloo on CPU): split roles reproduce colocated tokens.

BASELINE config #1: tiny DeepSeek-V2-style MoE, fp32, seed 0, 1 Attention +
1 FFN rank, 4 prompts x 32 uniform ids, 16 greedy tokens -> identical output.
"""

import pytest
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.launcher import LocalAFDSpec, launch_local


def _prompts(n=4, length=32, vocab=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g).tolist()


def _colocated(preset, prompts, max_tokens):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=128), max_num_seqs=8)
    m = build_model(arch, role="colocated", dtype=torch.float32, device="cpu", seed=0, max_positions=128)
    return LLMEngine(ec, m).generate(prompts, max_tokens)


def _run(preset, afd, prompts, max_tokens=16, **kw):
    res = launch_local(LocalAFDSpec(preset=preset, afd=afd, prompts=prompts, max_tokens=max_tokens, **kw))
    errs = {r: v for r, v in res.items() if "error" in v}
    assert not errs, errs
    outs = []
    for r in sorted(res):
        outs += res[r].get("outputs", [])
    return outs, res


def test_config1_1a1f_matches_colocated():
    prompts = _prompts()
    ref = _colocated("tiny-dsv2", prompts, 16)
    outs, res = _run("tiny-dsv2", {"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts)
    assert outs == ref
    assert res[0]["role"] == "ffn" and res[0]["steps"] == res[1]["steps"]


@pytest.mark.parametrize("A,F,gate", [(2, 1, False), (2, 2, False), (2, 1, True)])
def test_topologies_match_colocated(A, F, gate):
    prompts = _prompts(n=5)
    ref = _colocated("tiny-dsv2", prompts, 8)
    afd = {"num_attention_ranks": A, "num_ffn_ranks": F, "compute_gate_on_attention": gate}
    outs, _ = _run("tiny-dsv2", afd, prompts, max_tokens=8)
    assert outs == ref


def test_qwen3_moe_2a2f():
    prompts = _prompts(n=4, length=16)
    ref = _colocated("tiny-qwen3-moe", prompts, 6)
    outs, _ = _run("tiny-qwen3-moe", {"num_attention_ranks": 2, "num_ffn_ranks": 2}, prompts, max_tokens=6)
    assert outs == ref


def test_dbo_two_ubatches_matches():
    prompts = _prompts(n=4, length=16)
    ref = _colocated("tiny-dsv2", prompts, 6)
    outs, _ = _run("tiny-dsv2", {"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts, max_tokens=6,
                   use_ubatching=True)
    assert outs == ref


def test_qwen3_5_hybrid_2a1f():
    """Gated DeltaNet + gated attention on the Attention side, gated shared expert on the FFN side."""
    prompts = _prompts(n=4, length=12)
    ref = _colocated("tiny-qwen3.5", prompts, 6)
    outs, _ = _run("tiny-qwen3.5", {"num_attention_ranks": 2, "num_ffn_ranks": 1}, prompts, max_tokens=6)
    assert outs == ref


def test_dsv4_mhc_hash_routing_2a1f():
    """mHC streams stay on the Attention side; hash-routed layers ship the token ids to the FFN."""
    prompts = _prompts(n=4, length=12)
    ref = _colocated("tiny-dsv4", prompts, 6)
    outs, _ = _run("tiny-dsv4", {"num_attention_ranks": 2, "num_ffn_ranks": 1}, prompts, max_tokens=6)
    assert outs == ref


def test_dsv4_expert_parallel_2a2f():
    prompts = _prompts(n=4, length=12)
    ref = _colocated("tiny-dsv4", prompts, 5)
    outs, _ = _run("tiny-dsv4", {"num_attention_ranks": 2, "num_ffn_ranks": 2}, prompts, max_tokens=5)
    assert outs == ref


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3-moe"])
def test_attention_tp2_matches_colocated(preset):
    """Two Attention ranks as one DP rank with TP=2 (heads split, o_proj all-reduced) + 1 FFN rank."""
    prompts = _prompts(n=3, length=12)
    ref = _colocated(preset, prompts, 6)
    outs, _ = _run(preset, {"num_attention_ranks": 2, "num_ffn_ranks": 1}, prompts, max_tokens=6, tp=2)
    assert outs == ref


def test_dsv32_sparse_attention_2a2f():
    """DeepSeek sparse attention (indexer on the Attention side, prompts past index_topk) across 2A2F."""
    prompts = _prompts(n=4, length=20)
    ref = _colocated("tiny-dsv32", prompts, 6)
    outs, _ = _run("tiny-dsv32", {"num_attention_ranks": 2, "num_ffn_ranks": 2}, prompts, max_tokens=6)
    assert outs == ref


def test_dsv32_attention_tp2():
    """The indexer is replicated on both tensor-parallel ranks; the MLA heads are split."""
    prompts = _prompts(n=3, length=16)
    ref = _colocated("tiny-dsv32", prompts, 5)
    outs, _ = _run("tiny-dsv32", {"num_attention_ranks": 2, "num_ffn_ranks": 1}, prompts, max_tokens=5, tp=2)
    assert outs == ref


def test_deepseek_v1_mha_2a1f():
    """DeepSeek V1: multi-head attention on the Attention side, routed + shared experts on the FFN side."""
    prompts = _prompts(n=4, length=12)
    ref = _colocated("tiny-dsv1", prompts, 6)
    outs, _ = _run("tiny-dsv1", {"num_attention_ranks": 2, "num_ffn_ranks": 1}, prompts, max_tokens=6)
    assert outs == ref
