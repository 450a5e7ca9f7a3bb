"""Qwen3.5 / Qwen3-Next layers on CPU: checkpoint layouts, gates, roles, loading."""

import torch
import torch.nn.functional as F

from afd_plugin_b200.models import build_model, get_preset, weight_roles
from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.models.layers import AttentionMetadata, GatedDeltaNet, GatedGQAAttention
from afd_plugin_b200.ops import reference as ref

ARCH = get_preset("tiny-qwen3.5")


def _meta(T, slot=0):
    return AttentionMetadata(
        positions=torch.arange(T), slot_mapping=torch.arange(T), block_table=torch.zeros(1, 4, dtype=torch.int32),
        seq_lens=torch.tensor([T], dtype=torch.int32), is_decode=False, prefill_seqs=[(0, T, 0)],
        state_slots=torch.tensor([slot], dtype=torch.int32), cu_seqlens=torch.tensor([0, T], dtype=torch.int32),
        state_reset=torch.tensor([1], dtype=torch.int32))


def test_gdn_layer_matches_grouped_checkpoint_math():
    torch.manual_seed(0)
    a = ARCH
    la = GatedDeltaNet(a, torch.float32, "cpu")
    nk, nv, dk, dv, K = la.nk, la.nv, la.dk, la.dv, la.K
    r = nv // nk
    H = a.hidden_size
    w_qkvz = torch.randn(2 * la.key_dim + 2 * la.value_dim, H) * 0.05
    w_ba = torch.randn(2 * nv, H) * 0.2
    la.set_in_proj_qkvz(w_qkvz)
    la.set_in_proj_ba(w_ba)
    la.conv_weight.data.normal_(0, 0.3)
    la.A_log.data.normal_(0, 0.3)
    la.dt_bias.data.normal_(0, 0.3)
    la.norm_weight.data.fill_(1.0).add_(torch.randn(dv) * 0.1)
    la.out_proj.data.normal_(0, 0.05)
    T = 6
    x = torch.randn(T, H)
    conv_state = torch.zeros(2, la.conv_dim, K - 1)
    ssm_state = torch.zeros(2, nv, dk, dv)
    got = la(x, _meta(T, slot=1), (conv_state, ssm_state))

    # Independent statement of the layer from the checkpoint's grouped layout.
    qkvz = (x @ w_qkvz.t()).view(T, nk, 2 * dk + 2 * r * dv)
    q, k = qkvz[..., :dk], qkvz[..., dk : 2 * dk]
    v = qkvz[..., 2 * dk : 2 * dk + r * dv].reshape(T, nv, dv)
    z = qkvz[..., 2 * dk + r * dv :].reshape(T, nv, dv)
    ba = (x @ w_ba.t()).view(T, nk, 2 * r)
    b, aa = ba[..., :r].reshape(T, nv), ba[..., r:].reshape(T, nv)
    mixed = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], dim=-1)
    conv = F.conv1d(F.pad(mixed.t().unsqueeze(0), (K - 1, 0)), la.conv_weight.unsqueeze(1), groups=la.conv_dim)[0].t()
    conv = F.silu(conv)
    qc = conv[:, : nk * dk].view(T, nk, dk).repeat_interleave(r, 1)
    kc = conv[:, nk * dk : 2 * nk * dk].view(T, nk, dk).repeat_interleave(r, 1)
    vc = conv[:, 2 * nk * dk :].view(T, nv, dv)
    g = -la.A_log.exp() * F.softplus(aa + la.dt_bias)
    o, S = ref.gated_delta_rule(qc, kc, vc, g, torch.sigmoid(b))
    o = ref.rms_norm_gated(o, z, la.norm_weight, a.rms_norm_eps).reshape(T, -1)
    want = o @ la.out_proj.t()
    torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(ssm_state[1], S, atol=1e-5, rtol=1e-5)
    assert ssm_state[0].abs().sum() == 0  # other slots untouched


def test_gdn_prefill_then_decode_equals_one_prefill():
    torch.manual_seed(1)
    la = GatedDeltaNet(ARCH, torch.float32, "cpu")
    for p in la.parameters():
        p.data.normal_(0, 0.1)
    H = ARCH.hidden_size
    x = torch.randn(9, H)
    st_a = (torch.zeros(1, la.conv_dim, la.K - 1), torch.zeros(1, la.nv, la.dk, la.dv))
    full = la(x, _meta(9), st_a)
    st_b = (torch.zeros(1, la.conv_dim, la.K - 1), torch.zeros(1, la.nv, la.dk, la.dv))
    part = [la(x[:5], _meta(5), st_b)]
    for t in range(5, 9):
        m = AttentionMetadata(positions=torch.tensor([t]), slot_mapping=torch.tensor([t]),
                              block_table=torch.zeros(1, 4, dtype=torch.int32), seq_lens=torch.tensor([t + 1]),
                              is_decode=True, state_slots=torch.tensor([0], dtype=torch.int32),
                              cu_seqlens=torch.tensor([0, 1], dtype=torch.int32))
        part.append(la(x[t : t + 1], m, st_b))
    torch.testing.assert_close(torch.cat(part), full, atol=1e-5, rtol=1e-5)


def test_gated_attention_q_proj_interleave():
    torch.manual_seed(2)
    at = GatedGQAAttention(ARCH, torch.float32, "cpu")
    nq, d = at.nq, at.d
    w = torch.randn(2 * nq * d, ARCH.hidden_size)
    at.set_q_proj(w)
    per_head = w.view(nq, 2, d, -1)
    assert torch.equal(at.qkv_proj[: nq * d], per_head[:, 0].reshape(nq * d, -1))
    assert torch.equal(at.qkv_proj[nq * d : 2 * nq * d], per_head[:, 1].reshape(nq * d, -1))


def test_shared_expert_gate_scales_shared_output():
    torch.manual_seed(3)
    m = build_model(ARCH, role="colocated", dtype=torch.float32, seed=4)
    mlp = m.layers[0].mlp
    h = torch.randn(5, ARCH.hidden_size)
    w, ids = mlp.gate.route(mlp.gate.logits(h))
    routed = mlp.experts(h, w, ids)
    sg = torch.sigmoid(h @ mlp.shared_expert_gate.t())
    want = routed + sg * mlp.shared_experts(h)
    torch.testing.assert_close(mlp(h), want, atol=1e-5, rtol=1e-5)


def test_roles_and_norm_offsets():
    a = ARCH
    assert weight_roles("model.layers.0.linear_attn.in_proj_qkvz.weight", a, compute_gate_on_attention=False) == {
        "attention"}
    assert weight_roles("model.layers.3.self_attn.q_proj.weight", a, compute_gate_on_attention=False) == {"attention"}
    assert weight_roles("model.layers.1.mlp.shared_expert_gate.weight", a, compute_gate_on_attention=False) == {"ffn"}
    assert weight_roles("model.layers.1.mlp.shared_expert.up_proj.weight", a, compute_gate_on_attention=False) == {
        "ffn"}
    assert weight_roles("model.layers.1.mlp.gate.weight", a, compute_gate_on_attention=False,
                        route_on_attention=True) == {"attention", "ffn"}
    m = build_model(a, role="attention", dtype=torch.float32, seed=0)
    # zero-centred norms: checkpoint zeros load as weight 1
    assert torch.equal(m.layers[0].input_layernorm.weight, torch.ones(a.hidden_size))
    assert m.layers[0].mlp is None and m.layers[3].self_attn is not None


def test_from_hf_config_parses_hybrid_layout():
    hf = {"architectures": ["Qwen3NextForCausalLM"], "model_type": "qwen3_next", "hidden_size": 2048,
          "num_hidden_layers": 8, "vocab_size": 151936, "num_attention_heads": 16, "num_key_value_heads": 2,
          "head_dim": 256, "num_experts": 512, "num_experts_per_tok": 10, "moe_intermediate_size": 512,
          "shared_expert_intermediate_size": 512, "linear_num_key_heads": 16, "linear_num_value_heads": 32,
          "linear_key_head_dim": 128, "linear_value_head_dim": 128, "full_attention_interval": 4,
          "partial_rotary_factor": 0.25}
    a = ModelArchConfig.from_hf_config(hf)
    assert a.layer_types[3] == "full_attention" and a.layer_types[0] == "linear_attention"
    assert a.full_attention_layers == (3, 7) and a.rotary_dim == 64 and a.shared_expert_gate
    assert a.linear_conv_dim == 2 * 16 * 128 + 32 * 128


def test_multimodal_checkpoint_names_map_to_the_text_model():
    from afd_plugin_b200.models.loader import checkpoint_name

    assert checkpoint_name("model.language_model.layers.3.mlp.gate.weight") == "model.layers.3.mlp.gate.weight"
    assert checkpoint_name("model.visual.blocks.0.attn.qkv.weight") is None
    assert checkpoint_name("mtp.layers.0.mlp.gate.weight") is None
    assert checkpoint_name("lm_head.weight") == "lm_head.weight"
    assert checkpoint_name("model.embed_tokens.weight") == "model.embed_tokens.weight"


def test_multimodal_config_reads_text_config():
    text = {"model_type": "qwen3_5_moe_text", "hidden_size": 2048, "num_hidden_layers": 8, "vocab_size": 151936,
            "num_attention_heads": 16, "num_key_value_heads": 2, "head_dim": 256, "num_experts": 256,
            "num_experts_per_tok": 8, "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512,
            "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
            "linear_value_head_dim": 128, "full_attention_interval": 4, "eos_token_id": 248044}
    hf = {"architectures": ["Qwen3_5MoeForConditionalGeneration"], "model_type": "qwen3_5_moe",
          "text_config": text, "vision_config": {"depth": 27}}
    a = ModelArchConfig.from_hf_config(hf)
    assert a.architecture == "Qwen3_5MoeForConditionalGeneration" and a.hidden_size == 2048
    assert a.n_routed_experts == 256 and a.full_attention_layers == (3, 7) and a.eos_token_id == (248044,)
