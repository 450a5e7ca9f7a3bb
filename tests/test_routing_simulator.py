import pytest
import torch

from afd_plugin_b200.models.routing_simulator import balanced_topk, expert_cycle


def test_cycle_is_permutation_and_rotated():
    c0 = expert_cycle(16, 2, 0)
    c1 = expert_cycle(16, 2, 1)
    assert sorted(c0.tolist()) == list(range(16))
    assert torch.equal((c0 + 8) % 16, c1)


def test_topn_per_rank(monkeypatch):
    c = expert_cycle(16, 2, 0, topn_per_rank=2)
    assert c.tolist() == [0, 1, 8, 9]
    with pytest.raises(ValueError):
        expert_cycle(16, 2, 0, topn_per_rank=9)


def test_balanced_topk_uniform(monkeypatch):
    w, ids = balanced_topk(10, 8, 2, device="cpu")
    assert torch.allclose(w, torch.full((10, 2), 0.5))
    counts = torch.bincount(ids.flatten().long(), minlength=8)
    assert counts.max() - counts.min() <= 1


def test_gate_uses_balanced_routing(monkeypatch):
    from afd_plugin_b200.models import build_model, get_preset

    monkeypatch.setenv("AFD_FORCE_BALANCED_TOPK_IDS", "1")
    m = build_model(get_preset("tiny-dsv2"), dtype=torch.float32)
    gate = m.layers[1].mlp.gate
    w, ids = gate.route(torch.randn(5, 8))
    assert torch.allclose(w, torch.full_like(w, 0.5))
