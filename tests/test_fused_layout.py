"""Fused connector layout and options (CPU)."""

import pytest

from afd_plugin_b200.connectors.b200_fused import B200FusedExtraInfo, FusedLayout


def test_layout_sizes_6a2f():
    d = FusedLayout(num_attn=6, num_ffn=2, stages=1, layers=27, hidden=2048, experts=64, top_k=6, t_cap=43)
    assert d.ratio == 3 and d.e_local == 32 and d.cap == 258
    assert d.rows == 32 * 258 and d.slots == 7
    lay = d.heap_layout()
    assert lay["tok"].nbytes == 6 * 43 * 2048 * 2
    offs = sorted(r.offset for r in lay.regions.values())
    assert all(o % 256 == 0 for o in offs)
    assert lay.size < 64 * 2**20


def test_extra_config_strict():
    assert B200FusedExtraInfo.from_mapping({"max_tokens_per_rank": "64"}).max_tokens_per_rank == 64
    with pytest.raises(ValueError):
        B200FusedExtraInfo.from_mapping({"bogus": 1})
    with pytest.raises(ValueError):
        B200FusedExtraInfo.from_mapping({"wait_timeout_ms": 0})
    assert B200FusedExtraInfo.from_mapping({"fp8_dispatch": True}).fp8_dispatch
    with pytest.raises(TypeError):
        B200FusedExtraInfo.from_mapping({"fp8_dispatch": "maybe"})


def test_fp8_rows_halve_token_buffer():
    bf = FusedLayout(num_attn=6, num_ffn=2, stages=1, layers=27, hidden=2048, experts=64, top_k=6, t_cap=43)
    f8 = FusedLayout(num_attn=6, num_ffn=2, stages=1, layers=27, hidden=2048, experts=64, top_k=6, t_cap=43, fp8=True)
    lb, l8 = bf.heap_layout(), f8.heap_layout()
    assert l8["tok"].nbytes * 2 == lb["tok"].nbytes
    assert l8["tok_scale"].nbytes == 6 * 43 * 16 * 4 and "tok_scale" not in lb.regions
