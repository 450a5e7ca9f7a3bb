"""Deterministic, expert-parallel-balanced routing for performance runs.

Enabled by ``VLLM_MOE_ROUTING_SIMULATION_STRATEGY=afd_balanced`` (the name the
reference registers, ``afd_plugin/model_executor/routing_simulator.py:122-171``)
or ``AFD_FORCE_BALANCED_TOPK_IDS=1``.  Token ``t``'s ``j``-th expert is entry
``t * k + j`` of a cycle over the experts: either a seeded permutation of all
experts or, with ``AFD_BENCHMARK_FORCE_LB_TOPN_PER_RANK=n``, the first ``n``
experts of every expert-parallel rank.  The cycle is rotated by the rank's
first expert so ranks do not start on the same expert.  Weights are ``1/k``.
"""

from __future__ import annotations

import os
from functools import lru_cache

import torch

AFD_BALANCED = "afd_balanced"
_STRATEGY_ENV = "VLLM_MOE_ROUTING_SIMULATION_STRATEGY"
_TOPN_ENV = "AFD_BENCHMARK_FORCE_LB_TOPN_PER_RANK"
_SEED = 1024


def balanced_routing_enabled() -> bool:
    from afd_plugin_b200.envs import force_balanced_topk_ids_enabled

    return os.environ.get(_STRATEGY_ENV, "") == AFD_BALANCED or force_balanced_topk_ids_enabled()


def expert_cycle(num_experts: int, ep_size: int = 1, ep_rank: int = 0, topn_per_rank: int = 0) -> torch.Tensor:
    if num_experts <= 0 or ep_size <= 0 or not 0 <= ep_rank < ep_size or num_experts % ep_size:
        raise ValueError("invalid expert-parallel routing configuration")
    local = num_experts // ep_size
    if topn_per_rank:
        if not 0 < topn_per_rank <= local:
            raise ValueError(f"{_TOPN_ENV} must be between 1 and {local}")
        cyc = torch.cat([torch.arange(r * local, r * local + topn_per_rank, dtype=torch.int32)
                         for r in range(ep_size)])
    else:
        g = torch.Generator().manual_seed(_SEED)
        cyc = torch.randperm(num_experts, generator=g, dtype=torch.int32)
    return (cyc + ep_rank * local) % num_experts


@lru_cache(maxsize=32)
def _table(num_experts: int, top_k: int, tokens: int, ep_size: int, ep_rank: int, topn: int) -> torch.Tensor:
    cyc = expert_cycle(num_experts, ep_size, ep_rank, topn)
    if top_k > cyc.numel():
        raise ValueError("selected expert pool must contain at least top_k experts")
    total = tokens * top_k
    reps = (total + cyc.numel() - 1) // cyc.numel()
    return cyc.repeat(reps)[:total].view(tokens, top_k)


def balanced_topk(tokens: int, num_experts: int, top_k: int, *, device, ep_size: int = 1, ep_rank: int = 0,
                  token_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """``(weights fp32 [T, k], ids int32 [T, k])`` for ``tokens`` tokens."""
    topn = int(os.environ.get(_TOPN_ENV, "0") or 0)
    ids = _table(num_experts, top_k, token_offset + tokens, ep_size, ep_rank, topn)[token_offset:].to(device)
    w = torch.full((tokens, top_k), 1.0 / top_k, dtype=torch.float32, device=device)
    return w, ids


__all__ = ["AFD_BALANCED", "balanced_routing_enabled", "balanced_topk", "expert_cycle"]
