"""Token-count bookkeeping for the FFN role (CPU-only, no torch).

Same arithmetic as ``afd_plugin/v1/worker/ffn_metadata.py:8-69``: each FFN
rank's count is the sum of its ``r`` consecutive Attention peers, an empty
peer counts as one placeholder row, and counts given per DP rank are expanded
over TP peers first.
"""

from __future__ import annotations


def _expand_to_attention(counts: tuple[int, ...], attention_size: int) -> tuple[int, ...]:
    if counts and len(counts) < attention_size and attention_size % len(counts) == 0:
        per = attention_size // len(counts)
        return tuple(counts[i // per] for i in range(attention_size))
    return counts


def aggregate_ffn_token_counts(
    attention_counts: tuple[int, ...], *, attention_size: int, ffn_size: int, fallback: int = 1
) -> tuple[int, ...]:
    fb = max(1, int(fallback))
    if ffn_size <= 0 or attention_size < ffn_size or attention_size % ffn_size:
        return tuple(fb for _ in range(max(0, ffn_size)))
    counts = _expand_to_attention(tuple(attention_counts), attention_size)
    r = attention_size // ffn_size
    out = []
    for f in range(ffn_size):
        total = 0
        for a in range(f * r, (f + 1) * r):
            total += max(1, int(counts[a])) if a < len(counts) else fb
        out.append(total)
    return tuple(out)


def project_ffn_token_counts_to_dp(ffn_counts: tuple[int, ...], *, dp_size: int) -> tuple[int, ...]:
    if dp_size <= 0 or len(ffn_counts) == dp_size or len(ffn_counts) % dp_size:
        return tuple(ffn_counts)
    per = len(ffn_counts) // dp_size
    return tuple(ffn_counts[d * per] for d in range(dp_size))


__all__ = ["aggregate_ffn_token_counts", "project_ffn_token_counts_to_dp"]
