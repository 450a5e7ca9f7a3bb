"""AFD over real processes (gloo on CPU): split roles reproduce colocated tokens.

Correctness oracle: tiny DeepSeek-V2-style MoE, fp32, seed 0, 1 Attention +
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


def test_config1_1a1f_logits_match_colocated():
    """The Attention rank's logits of the prefill and first decode step equal the
    colocated model's (fp32, same ops on both sides)."""
    prompts = _prompts()
    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=128), max_num_seqs=8)
    eng = LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, device="cpu", seed=0,
                                    max_positions=128))
    for p in prompts:
        eng.add_request(p, 4)
    ref = []
    for _ in range(2):
        eng.step()
        ref.append(eng.runner.last_logits[: len(prompts)].float())
    _, res = _run("tiny-dsv2", {"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts, max_tokens=4,
                  record_logits_steps=2)
    got = [torch.from_numpy(a) for a in res[1]["logits"]]
    assert len(got) == 2
    for g, r in zip(got, ref):
        torch.testing.assert_close(g, r, atol=1e-5, rtol=1e-5)


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


@pytest.mark.parametrize("async_scheduling", [False, True], ids=["sync", "async"])
def test_dbo_two_ubatches_matches(async_scheduling):
    prompts = _prompts(n=4, length=16)
    ref = _colocated("tiny-dsv2", prompts, 6)
    outs, _ = _run("tiny-dsv2", {"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts, max_tokens=6,
                   use_ubatching=True, async_scheduling=async_scheduling)
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


@pytest.mark.parametrize("async_scheduling", [False, True], ids=["sync", "async"])
def test_dsv32_sparse_attention_2a2f(async_scheduling):
    """DeepSeek sparse attention (indexer on the Attention side, prompts past index_topk) across 2A2F;
    with async scheduling the ranks agree on the sparse mode in the same exchange as the launch sizes."""
    prompts = _prompts(n=4, length=20)
    ref = _colocated("tiny-dsv32", prompts, 6)
    outs, res = _run("tiny-dsv32", {"num_attention_ranks": 2, "num_ffn_ranks": 2}, prompts, max_tokens=6,
                     async_scheduling=async_scheduling)
    assert outs == ref
    if async_scheduling:
        assert all(v["async_steps"] >= 3 for v in res.values() if v["role"] == "attention")


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


def test_afd_from_an_hf_checkpoint(tmp_path):
    """Architecture from config.json, role-filtered weights from safetensors, on every rank."""
    import json as _json
    import zlib

    from safetensors.torch import save_file

    from afd_plugin_b200.models.loader import read_hf_config

    a = get_preset("tiny-dsv2")
    hf = {"architectures": ["DeepseekV2ForCausalLM"], "model_type": "deepseek_v2", "hidden_size": a.hidden_size,
          "num_hidden_layers": a.num_hidden_layers, "vocab_size": a.vocab_size,
          "num_attention_heads": a.num_attention_heads, "q_lora_rank": a.q_lora_rank,
          "kv_lora_rank": a.kv_lora_rank, "qk_nope_head_dim": a.qk_nope_head_dim,
          "qk_rope_head_dim": a.qk_rope_head_dim, "v_head_dim": a.v_head_dim,
          "intermediate_size": a.intermediate_size, "first_k_dense_replace": a.first_k_dense_replace,
          "n_routed_experts": a.n_routed_experts, "num_experts_per_tok": a.num_experts_per_tok,
          "moe_intermediate_size": a.moe_intermediate_size, "n_shared_experts": a.n_shared_experts,
          "scoring_func": a.scoring_func, "topk_method": a.topk_method, "n_group": a.n_group,
          "topk_group": a.topk_group, "norm_topk_prob": a.norm_topk_prob,
          "routed_scaling_factor": a.routed_scaling_factor, "max_position_embeddings": 2048}
    (tmp_path / "config.json").write_text(_json.dumps(hf))
    parsed = read_hf_config(str(tmp_path))
    src = build_model(parsed, role="colocated", dtype=torch.float32, seed=0)
    tensors = {}
    for spec in src.param_specs():
        g = torch.Generator().manual_seed(zlib.crc32(spec.name.encode()) & 0xFFFF)
        t = torch.randn(spec.shape, generator=g) * 0.05
        if spec.init == "ones":
            t = 1.0 + t * 0.1
        tensors[spec.name] = t
    save_file(tensors, str(tmp_path / "model.safetensors"))
    prompts = _prompts(n=3, length=10)
    ec = EngineConfig(ModelConfig(parsed, dtype=torch.float32, enforce_eager=True, max_model_len=128,
                                  checkpoint=str(tmp_path)), max_num_seqs=8)
    ref = LLMEngine(ec, build_model(parsed, role="colocated", dtype=torch.float32, checkpoint=str(tmp_path),
                                    max_positions=128)).generate(prompts, 5)
    res = launch_local(LocalAFDSpec(preset=None, checkpoint=str(tmp_path), prompts=prompts, max_tokens=5,
                                    afd={"num_attention_ranks": 2, "num_ffn_ranks": 1}))
    assert not any("error" in v for v in res.values()), res
    outs = []
    for r in sorted(res):
        outs += res[r].get("outputs", [])
    assert outs == ref


@pytest.mark.parametrize("A,F,tp", [(1, 1, 1), (2, 1, 1), (2, 2, 1), (2, 1, 2)])
def test_async_scheduling_matches_colocated(A, F, tp):
    """Decode steps launched before the previous step's tokens are read (uneven DP shares pad to the
    largest rank's batch) give the colocated tokens."""
    prompts = _prompts(n=5, length=12)
    ref = _colocated("tiny-dsv2", prompts, 7)
    outs, res = _run("tiny-dsv2", {"num_attention_ranks": A, "num_ffn_ranks": F}, prompts, max_tokens=7, tp=tp,
                     async_scheduling=True)
    assert outs == ref
    assert all(v["async_steps"] >= 4 for v in res.values() if v["role"] == "attention")
