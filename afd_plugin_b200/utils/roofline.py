"""Bytes a decode step must move through HBM, and the bandwidth roofline they imply.

A decode step reads every weight it uses once (tokens reuse each weight tile
in on-chip memory) and every cached KV row of the running sequences once per
attention layer; the activations are small next to both.  So the
memory-bound lower limit of a step is ``(weight bytes + KV bytes) / HBM
bandwidth``, and ``achieved = bytes / step time`` divided by the measured
copy bandwidth is the step's roofline fraction.

The embedding table is excluded (a step gathers one row per token); a tied
LM head counts once, as the head.  The measured bandwidth comes from
``MEASURED_PEAKS.json`` at the repository root when present (a STREAM-style
copy on this machine's GPUs), else a fallback figure for B200.
"""

from __future__ import annotations

import json
import os

FALLBACK_HBM_GBS = 6650.0


def hbm_peak_gbs() -> tuple[float, str]:
    """(GB/s, "measured" | "fallback")."""
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError, TypeError):
        return FALLBACK_HBM_GBS, "fallback"


def weight_bytes_per_step(model) -> int:
    """Bytes of this rank's parameters a decode step reads (the embedding gather excluded)."""
    embed = getattr(model, "embed_tokens", None)
    head = getattr(model, "lm_head", None)
    skip = {id(embed)} if embed is not None and embed is not head else set()
    seen: set[int] = set()
    total = 0
    for p in model.parameters():
        if id(p) in skip or p.data_ptr() in seen:
            continue
        seen.add(p.data_ptr())
        total += p.numel() * p.element_size()
    return total


def kv_bytes_per_step(arch, context_tokens: int, *, elem_bytes: int = 2) -> int:
    """Cache bytes read by one decode step over ``context_tokens`` cached positions in total."""
    layers = len(arch.full_attention_layers)
    return int(context_tokens) * arch.kv_cache_width * elem_bytes * layers


__all__ = ["FALLBACK_HBM_GBS", "hbm_peak_gbs", "kv_bytes_per_step", "weight_bytes_per_step"]
