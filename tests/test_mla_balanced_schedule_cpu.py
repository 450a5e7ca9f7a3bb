"""The work-balanced MLA decode schedule, restated in fp32 PyTorch.

``ops/csrc/mla_decode.cu::mla_decode_bal_kernel`` lays the requests' 32-token
tiles end to end (request b owns global tiles [P_b, P_{b+1}), at least one
tile each), gives CTA c the tiles [c W, (c + 1) W) with W = ceil(P_B / C),
writes a request that one CTA covers directly, and otherwise merges the
covering CTAs' partials from slot 2 c (the request is the CTA's first
segment) or 2 c + 1.  This test runs the same formulas on the host and checks
that every request's merged output equals plain attention over its context,
for CTA counts below, at and above the tile count.
"""

from __future__ import annotations

import math

import pytest
import torch

TILE = 32


def _schedule(seq_lens: list[int], ctas: int):
    tiles = [max(1, math.ceil(s / TILE)) for s in seq_lens]
    prefix = [0]
    for t in tiles:
        prefix.append(prefix[-1] + t)
    total = prefix[-1]
    w = math.ceil(total / ctas)
    return prefix, total, w


def _segments(prefix, w, total, c):
    """(request, first tile, end tile, segment index) of CTA c, as the kernel walks them."""
    g0, g1 = c * w, min(total, c * w + w)
    if g0 >= g1:
        return []
    b = max(i for i in range(len(prefix) - 1) if prefix[i] <= g0)  # the kernel's binary search
    out, seg = [], 0
    while b < len(prefix) - 1 and prefix[b] < g1:
        p0 = prefix[b]
        out.append((b, max(g0, p0) - p0, min(g1, prefix[b + 1]) - p0, seg))
        b += 1
        seg += 1
    return out


def _partial(q, kv, seq, t_lo, t_hi, scale):
    """Normalised partial output and log2-sum-exp of q [H, D] over tiles [t_lo, t_hi) of kv [S, D]."""
    lo, hi = t_lo * TILE, t_hi * TILE
    s = (q @ kv[lo:hi].T) * scale * math.log2(math.e)  # exp2 domain, as the kernel
    tok = torch.arange(lo, hi)
    s = s.masked_fill(tok[None, :] >= seq, float("-inf"))
    m = s.max(dim=1, keepdim=True).values
    m_use = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    p = torch.exp2(s - m_use)
    l = p.sum(dim=1, keepdim=True)
    o = (p @ kv[lo:hi, :512]) / torch.where(l > 0, l, torch.ones_like(l))
    lse = torch.where(l > 0, m_use + torch.log2(l), torch.full_like(l, float("-inf")))
    return o, lse.squeeze(1)


def _run(seq_lens, ctas, heads=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    D, scale = 576, 0.1
    qs = [torch.randn(heads, D, generator=g) for _ in seq_lens]
    kvs = [torch.randn(max(1, math.ceil(s / TILE)) * TILE, D, generator=g) for s in seq_lens]
    prefix, total, w = _schedule(seq_lens, ctas)
    part_o, part_lse, out = {}, {}, {}
    arrivals = [0] * len(seq_lens)
    for c in range(ctas):
        for b, t_lo, t_hi, seg in _segments(prefix, w, total, c):
            o, lse = _partial(qs[b], kvs[b], seq_lens[b], t_lo, t_hi, scale)
            first_cta = prefix[b] // w
            n_chunks = (prefix[b + 1] - 1) // w - first_cta + 1
            if n_chunks == 1:
                out[b] = o
                continue
            slot = c * 2 + (0 if seg == 0 else 1)
            assert slot not in part_o  # no two chunks share a slot
            part_o[slot], part_lse[slot] = o, lse
            arrivals[b] += 1
            if arrivals[b] == n_chunks:  # the last chunk merges
                second = prefix[b] != first_cta * w
                slots = [(first_cta + j) * 2 + (1 if (j == 0 and second) else 0) for j in range(n_chunks)]
                lses = torch.stack([part_lse[s] for s in slots])  # [n, H]
                mx = lses.max(dim=0).values
                wts = torch.where(torch.isinf(lses), torch.zeros_like(lses), torch.exp2(lses - mx))
                wts = wts / wts.sum(dim=0).clamp_min(1e-30)
                out[b] = sum(wts[j][:, None] * part_o[s] for j, s in enumerate(slots))
    assert sorted(out) == list(range(len(seq_lens)))  # every request written exactly once
    for b, s in enumerate(seq_lens):
        if s == 0:
            assert torch.count_nonzero(out[b]) == 0
            continue
        ref = torch.softmax((qs[b] @ kvs[b][:s].T) * scale, dim=1) @ kvs[b][:s, :512]
        torch.testing.assert_close(out[b], ref, atol=2e-5, rtol=2e-5)
    return w


@pytest.mark.parametrize("seq_lens,ctas", [
    ([1034] * 12, 10),              # every CTA crosses a request boundary
    ([1034] * 4, 37),               # each request over several CTAs; some CTAs start inside a request
    ([5000], 296),                  # one long request over every CTA (157 tiles: most CTAs idle past W)
    ([40, 3000, 7, 64, 65, 999, 1], 9),
    ([64, 64, 64, 64], 4),          # requests start exactly on CTA boundaries
    ([0, 33, 0, 100], 3),           # empty requests: one masked tile, zero output
    ([31, 32, 33], 50),             # more CTAs than tiles
])
def test_balanced_schedule_reproduces_attention(seq_lens, ctas):
    _run(seq_lens, ctas)


def test_bench_shape_balances_the_wave():
    """256 requests of 1034 tokens on 296 CTAs: 29 tiles per CTA instead of one 33-tile request each."""
    prefix, total, w = _schedule([1034] * 256, 296)
    assert total == 256 * 33 and w == 29
    loads = [sum(hi - lo for _, lo, hi, _ in _segments(prefix, w, total, c)) for c in range(296)]
    assert max(loads) == 29 and sum(loads) == total
