"""Model zoo on CPU: KV-cached decode matches full recompute, role splits, loading."""

import json
import os

import pytest
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import MODEL_REGISTRY, build_model, get_preset, weight_roles
from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.models.loader import load_weights
from afd_plugin_b200.runtime.engine import LLMEngine

PRESETS = ["tiny-dsv2", "tiny-qwen3-moe", "tiny-dsv3", "tiny-qwen3.5", "tiny-dsv4", "tiny-dsv1", "tiny-dsv32"]


def _engine(preset, **kw):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96), max_num_seqs=4)
    m = build_model(arch, role="colocated", dtype=torch.float32, device="cpu", seed=0, max_positions=96, **kw)
    return LLMEngine(ec, m)


@pytest.mark.parametrize("preset", PRESETS)
def test_decode_matches_full_recompute(preset):
    eng = _engine(preset)
    g = torch.Generator().manual_seed(1)
    vocab = eng.model.arch.vocab_size
    prompts = torch.randint(0, vocab, (3, 10), generator=g).tolist()
    outs = eng.generate(prompts, 6)
    # Re-run each prefix as one prefill: every next token must agree.
    from afd_plugin_b200.runtime.engine import Request

    for p, o in zip(prompts, outs):
        seq = p + o[:-1]
        got = []
        for cut in range(len(p), len(seq) + 1):
            f2 = _engine(preset)
            req = Request(0, seq[:cut], 1)
            f2._ensure_blocks(req, cut + 1)
            got.append(int(f2.runner.prefill([seq[:cut]], [req.blocks], [0])[0]))
        assert got == o


def test_decode_batch_equals_single():
    eng = _engine("tiny-dsv2")
    g = torch.Generator().manual_seed(2)
    prompts = torch.randint(0, 1024, (4, 12), generator=g).tolist()
    batch = eng.generate(prompts, 5)
    singles = [_engine("tiny-dsv2").generate([p], 5)[0] for p in prompts]
    assert batch == singles


def test_role_weights_split():
    arch = get_preset("tiny-dsv2")
    assert weight_roles("model.layers.0.self_attn.q_proj.weight", arch, compute_gate_on_attention=False) == {"attention"}
    assert weight_roles("model.layers.0.mlp.gate_proj.weight", arch, compute_gate_on_attention=False) == {"ffn"}
    assert weight_roles("model.layers.0.mlp.gate_proj.weight", arch, compute_gate_on_attention=True) == {"attention"}
    assert weight_roles("model.layers.1.mlp.gate.weight", arch, compute_gate_on_attention=True) == {"attention", "ffn"}
    assert weight_roles("model.layers.1.mlp.experts.3.up_proj.weight", arch, compute_gate_on_attention=True) == {"ffn"}
    assert weight_roles("model.embed_tokens.weight", arch, compute_gate_on_attention=False) == {"attention", "ffn"}


def test_split_roles_hold_identical_weights():
    arch = get_preset("tiny-dsv2")
    full = build_model(arch, role="colocated", dtype=torch.float32, seed=3)
    attn = build_model(arch, role="attention", dtype=torch.float32, seed=3)
    ffn1 = build_model(arch, role="ffn", dtype=torch.float32, seed=3, ep_rank=1, ep_size=2)
    assert torch.equal(full.layers[0].self_attn.q_proj, attn.layers[0].self_attn.q_proj)
    assert torch.equal(full.layers[1].mlp.experts.w13[4:], ffn1.layers[1].mlp.experts.w13)
    assert ffn1.layers[0].self_attn is None and attn.layers[1].mlp is None


def test_load_from_safetensors_roundtrip(tmp_path):
    from safetensors.torch import save_file

    arch = get_preset("tiny-qwen3-moe")
    src = build_model(arch, role="colocated", dtype=torch.float32, seed=5)
    tensors = {}
    for spec in src.param_specs():
        gen = torch.Generator().manual_seed(hash(spec.name) & 0xFFFF)
        tensors[spec.name] = torch.randn(spec.shape, generator=gen) * 0.02
    save_file(tensors, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe", "hidden_size": arch.hidden_size,
        "num_hidden_layers": arch.num_hidden_layers, "vocab_size": arch.vocab_size,
        "num_attention_heads": arch.num_attention_heads, "num_key_value_heads": arch.num_key_value_heads,
        "head_dim": arch.head_dim, "num_experts": arch.n_routed_experts,
        "num_experts_per_tok": arch.num_experts_per_tok, "moe_intermediate_size": arch.moe_intermediate_size,
        "max_position_embeddings": 2048}))
    from afd_plugin_b200.models.loader import read_hf_config

    parsed = read_hf_config(str(tmp_path))
    assert parsed.attention_type == "gqa" and parsed.n_routed_experts == arch.n_routed_experts
    ffn = build_model(parsed, role="ffn", dtype=torch.float32, checkpoint=str(tmp_path), ep_rank=1, ep_size=2)
    e = parsed.n_routed_experts // 2
    assert torch.equal(ffn.layers[0].mlp.experts.w2[0], tensors[f"model.layers.0.mlp.experts.{e}.down_proj.weight"])
    attn = build_model(parsed, role="attention", dtype=torch.float32, checkpoint=str(tmp_path))
    q = tensors["model.layers.1.self_attn.k_proj.weight"]
    nq = parsed.num_attention_heads * parsed.head_dim
    assert torch.equal(attn.layers[1].self_attn.qkv_proj[nq: nq + q.shape[0]], q)


def test_fp8_block_weights_random_init():
    arch = get_preset("tiny-dsv3").scaled(quant="fp8_block")
    m = build_model(arch, role="ffn", dtype=torch.float32, seed=0)
    ex = m.layers[1].mlp.experts
    assert ex.w13.dtype == torch.float8_e4m3fn and ex.w13_scale.shape == (ex.n_local, 2, 2)
    from afd_plugin_b200.ops.reference import dequant_block

    w = dequant_block(ex.w13[0], ex.w13_scale[0])
    assert w.abs().max() < 0.2 and w.std() > 0.01


def test_registry_aliases():
    assert MODEL_REGISTRY["AFDDeepseekV2ForCausalLM"] is MODEL_REGISTRY["DeepseekV2ForCausalLM"]
    assert "AFDQwen3MoeForCausalLM" in MODEL_REGISTRY


def test_qwen_rejects_gate_on_attention():
    with pytest.raises(ValueError):
        build_model(get_preset("tiny-qwen3-moe"), role="attention", compute_gate_on_attention=True)


def test_hf_config_parse_dsv3():
    hf = {"architectures": ["DeepseekV3ForCausalLM"], "model_type": "deepseek_v3", "hidden_size": 7168,
          "num_hidden_layers": 61, "vocab_size": 129280, "num_attention_heads": 128, "q_lora_rank": 1536,
          "kv_lora_rank": 512, "qk_nope_head_dim": 128, "qk_rope_head_dim": 64, "v_head_dim": 128,
          "intermediate_size": 18432, "first_k_dense_replace": 3, "n_routed_experts": 256,
          "num_experts_per_tok": 8, "moe_intermediate_size": 2048, "n_shared_experts": 1,
          "scoring_func": "sigmoid", "topk_method": "noaux_tc", "n_group": 8, "topk_group": 4,
          "norm_topk_prob": True, "routed_scaling_factor": 2.5,
          "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128]}}
    a = ModelArchConfig.from_hf_config(hf)
    assert a.quant == "fp8_block" and a.is_moe_layer(3) and not a.is_moe_layer(2) and a.n_group == 8


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3.5", "tiny-dsv4"])
def test_reload_weights_in_place(preset):
    arch = get_preset(preset)
    m = build_model(arch, role="colocated", dtype=torch.float32, seed=1)
    ptrs = [p.data_ptr() for p in m.parameters()]
    m.reload_weights(seed=2)
    assert [p.data_ptr() for p in m.parameters()] == ptrs
    fresh = build_model(arch, role="colocated", dtype=torch.float32, seed=2)
    for (n, a), (_, b) in zip(m.named_parameters(), fresh.named_parameters()):
        assert torch.equal(a, b), n
    moe = next(l.mlp for l in m.layers if hasattr(l.mlp, "experts"))
    if moe.gate is not None:
        assert torch.equal(moe.gate.weight_f32, fresh_gate(fresh).weight_f32)


def fresh_gate(model):
    return next(l.mlp for l in model.layers if hasattr(l.mlp, "experts")).gate



def test_reload_weights_from_checkpoint_on_split_roles(tmp_path):
    from safetensors.torch import save_file

    arch = get_preset("tiny-dsv2")
    src = build_model(arch, role="colocated", dtype=torch.float32, seed=7)
    tensors = {}
    for spec in src.param_specs():
        gen = torch.Generator().manual_seed(zlib_crc(spec.name))
        tensors[spec.name] = torch.randn(spec.shape, generator=gen) * 0.02
    save_file(tensors, str(tmp_path / "model.safetensors"))
    ffn = build_model(arch, role="ffn", dtype=torch.float32, seed=0, ep_rank=1, ep_size=2)
    ptrs = [p.data_ptr() for p in ffn.parameters()]
    ffn.reload_weights(str(tmp_path))
    assert [p.data_ptr() for p in ffn.parameters()] == ptrs
    ref = build_model(arch, role="ffn", dtype=torch.float32, checkpoint=str(tmp_path), ep_rank=1, ep_size=2)
    for (n, a), (_, b) in zip(ffn.named_parameters(), ref.named_parameters()):
        assert torch.equal(a, b), n
    # packed shared-expert slots follow the reloaded shared expert
    ex = ffn.layers[1].mlp.experts
    assert torch.equal(ex.w13_all[ex.n_local:], ref.layers[1].mlp.experts.w13_all[ex.n_local:])


def zlib_crc(name: str) -> int:
    import zlib

    return zlib.crc32(name.encode()) & 0xFFFF


def test_deepseek_v1_config_is_multi_head_attention():
    hf = {"architectures": ["DeepseekForCausalLM"], "model_type": "deepseek", "hidden_size": 2048,
          "num_hidden_layers": 28, "vocab_size": 102400, "num_attention_heads": 16, "num_key_value_heads": 16,
          "intermediate_size": 10944, "moe_intermediate_size": 1408, "n_routed_experts": 64,
          "num_experts_per_tok": 6, "n_shared_experts": 2, "first_k_dense_replace": 1, "moe_layer_freq": 1,
          "scoring_func": "softmax", "norm_topk_prob": False}
    a = ModelArchConfig.from_hf_config(hf)
    assert a.attention_type == "gqa" and a.head_dim == 128 and not a.qk_norm
    assert MODEL_REGISTRY[a.architecture].__name__ == "AFDDeepseekForCausalLM"
    assert a == get_preset("deepseek-moe-16b").scaled(rope_scaling=None)
    m = build_model(get_preset("tiny-dsv1"), role="attention", dtype=torch.float32, seed=0)
    names = {s.name for s in m.param_specs()}
    assert "model.layers.1.self_attn.k_proj.weight" in names and not any("q_norm" in n for n in names)


def test_fp8_checkpoint_attention_weights_are_dequantised(tmp_path):
    """DeepSeek-V3 fp8 checkpoints store attention projections as e4m3 + weight_scale_inv too."""
    import zlib

    from safetensors.torch import save_file

    from afd_plugin_b200.ops.reference import dequant_block, quant_fp8_block_weight

    arch = get_preset("tiny-dsv3").scaled(quant="fp8_block")
    src = build_model(arch, role="colocated", dtype=torch.float32, seed=0)
    tensors, want = {}, {}
    for spec in src.param_specs():
        g = torch.Generator().manual_seed(zlib.crc32(spec.name.encode()) & 0xFFFF)
        w = torch.randn(spec.shape, generator=g) * 0.05
        if len(spec.shape) == 2 and "self_attn" in spec.name and "norm" not in spec.name:
            q, s = quant_fp8_block_weight(w)
            tensors[spec.name], tensors[spec.name + "_scale_inv"] = q, s
            want[spec.name] = dequant_block(q, s)
        elif spec.fp8_scale_name:
            q, s = quant_fp8_block_weight(w)
            tensors[spec.name], tensors[spec.fp8_scale_name] = q, s
        else:
            tensors[spec.name] = w
    save_file(tensors, str(tmp_path / "model.safetensors"))
    m = build_model(arch, role="attention", dtype=torch.float32, checkpoint=str(tmp_path))
    attn = m.layers[1].self_attn
    q_a = want["model.layers.1.self_attn.q_a_proj.weight"]
    assert torch.allclose(attn.in_proj[: q_a.shape[0]], q_a)
    assert torch.allclose(attn.o_proj, want["model.layers.1.self_attn.o_proj.weight"])
    del tensors["model.layers.1.self_attn.o_proj.weight_scale_inv"]
    save_file(tensors, str(tmp_path / "model.safetensors"))
    with pytest.raises(ValueError, match="weight_scale_inv"):
        build_model(arch, role="attention", dtype=torch.float32, checkpoint=str(tmp_path))


def test_rope_scaling_kinds():
    from afd_plugin_b200.ops.reference import rope_cos_sin_cache

    plain = rope_cos_sin_cache(8, 16, 10000.0)
    lin = rope_cos_sin_cache(8, 16, 10000.0, {"type": "linear", "factor": 2.0})
    # linear interpolation: position p with factor 2 rotates like position p / 2
    assert torch.allclose(lin[6], plain[3], atol=1e-6)
    assert torch.equal(rope_cos_sin_cache(8, 16, 10000.0, {"rope_type": "default"}), plain)
    with pytest.raises(ValueError, match="unsupported rope_scaling"):
        rope_cos_sin_cache(8, 16, 10000.0, {"type": "dynamic", "factor": 2.0})


def test_tied_word_embeddings_share_the_table(tmp_path):
    from safetensors.torch import save_file

    arch = get_preset("tiny-qwen3-moe").scaled(tie_word_embeddings=True)
    m = build_model(arch, role="colocated", dtype=torch.float32, seed=0)
    assert m.lm_head is m.embed_tokens
    names = [s.name for s in m.param_specs()]
    assert "lm_head.weight" not in names
    save_file({s.name: torch.randn(s.shape) * 0.02 for s in m.param_specs()}, str(tmp_path / "model.safetensors"))
    loaded = build_model(arch, role="attention", dtype=torch.float32, checkpoint=str(tmp_path))
    assert torch.equal(loaded.lm_head, loaded.embed_tokens)
    eng_out = LLMEngine(EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64),
                                     max_num_seqs=2), m).generate([[1, 2, 3]], 3)
    assert len(eng_out[0]) == 3
