"""DeepSeek-V4 family on CPU: mHC mixing, hash routing, roles, AFD split parity."""

import torch

from afd_plugin_b200.models import build_model, get_preset, weight_roles
from afd_plugin_b200.models.configs import ModelArchConfig
from afd_plugin_b200.ops import reference as ref

ARCH = get_preset("tiny-dsv4")


def test_mhc_residual_mixing_is_doubly_stochastic():
    torch.manual_seed(0)
    T, n, H = 5, ARCH.hc_mult, 32
    streams = torch.randn(T, n, H)
    fn = torch.randn((2 + n) * n, n * H) * 0.1
    base = torch.randn((2 + n) * n) * 0.1
    pre, post, res = ref.mhc_mix(streams, fn, base, torch.ones(3), norm_eps=1e-6, hc_eps=1e-6, post_alpha=2.0,
                                 sinkhorn_iters=20)
    torch.testing.assert_close(res.sum(-1), torch.ones(T, n), atol=1e-4, rtol=0)
    torch.testing.assert_close(res.sum(-2), torch.ones(T, n), atol=1e-4, rtol=0)
    assert bool((pre > 0).all() and (pre < 1.01).all() and (post > 0).all() and (post < 2).all())
    # identity mixing with zero post keeps the streams
    out = ref.mhc_post(streams, torch.zeros(T, H), torch.zeros(T, n), torch.eye(n).expand(T, n, n))
    torch.testing.assert_close(out, streams)


def test_hash_routing_uses_token_table():
    torch.manual_seed(1)
    m = build_model(ARCH, role="colocated", dtype=torch.float32, seed=2)
    gate = m.layers[1].mlp.gate  # hash layer
    assert gate.tid2eid is not None and m.layers[2].mlp.gate.tid2eid is None
    ids = torch.tensor([3, 3, 17, 900])
    h = torch.randn(4, ARCH.hidden_size)
    w, e = gate.route(gate.logits(h), ids)
    assert torch.equal(e.long(), gate.tid2eid[ids.long()].long())
    scores = torch.sqrt(torch.nn.functional.softplus(gate.logits(h)))
    g = scores.gather(1, e.long())
    torch.testing.assert_close(w, g / g.sum(-1, keepdim=True) * ARCH.routed_scaling_factor)


def test_v4_roles():
    a = ARCH
    r = lambda n, **k: weight_roles(n, a, compute_gate_on_attention=False, **k)  # noqa: E731
    assert r("model.layers.1.ffn.experts.3.up_proj.weight") == {"ffn"}
    assert r("model.layers.1.ffn.gate.tid2eid") == {"ffn"}
    assert r("model.layers.1.ffn.gate.weight", route_on_attention=True) == {"attention", "ffn"}
    assert r("model.layers.1.attn.kv_b_proj.weight") == {"attention"}
    assert r("model.layers.1.hc_ffn_fn") == {"attention"}
    assert r("model.hc_head_fn") == {"attention"}
    assert r("model.embed_tokens.weight") == {"attention", "ffn"}
    ffn = build_model(a, role="ffn", dtype=torch.float32, seed=0)
    attn = build_model(a, role="attention", dtype=torch.float32, seed=0)
    assert ffn.layers[1].mlp.gate.tid2eid is not None and not hasattr(ffn.layers[1], "hc_attn_fn")
    assert attn.layers[1].mlp is None and attn.layers[1].hc_ffn_fn.shape == ((2 + 4) * 4, 4 * a.hidden_size)


def test_v4_from_hf_config():
    hf = {"architectures": ["DeepseekV4ForCausalLM"], "hidden_size": 1024, "num_hidden_layers": 4, "vocab_size": 4096,
          "num_attention_heads": 8, "q_lora_rank": 256, "kv_lora_rank": 512, "qk_nope_head_dim": 128,
          "qk_rope_head_dim": 64, "v_head_dim": 128, "n_routed_experts": 64, "num_experts_per_tok": 6,
          "moe_intermediate_size": 512, "n_shared_experts": 1, "hc_mult": 4, "num_hash_layers": 3}
    a = ModelArchConfig.from_hf_config(hf)
    assert a.architecture == "DeepseekV4ForCausalLM" and a.hc_mult == 4 and a.scoring_func == "sqrtsoftplus"
    assert a.num_hash_layers == 3 and a.hc_sinkhorn_iters == 20
