"""sm_100a kernels vs the plain PyTorch fp32 reference of the same op."""

import math

import os

import pytest
import torch

from afd_plugin_b200 import ops
from afd_plugin_b200.ops import _ext
from afd_plugin_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(a, b, atol, rtol=0.0):
    torch.testing.assert_close(a.float().cpu(), b.float().cpu(), atol=atol, rtol=rtol)


@pytest.fixture(autouse=True)
def _status_clean():
    C = _ext.ops()
    C.reset_status(0)
    yield
    torch.cuda.synchronize()
    assert C.read_status(0) == 0, "a kernel wait timed out"


def test_extension_loaded_from_tree():
    assert _ext.load() and _ext.loaded_path().endswith(".so")


@pytest.mark.parametrize("hidden", [128, 512, 2048, 7168])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rms_norm(hidden, dtype):
    x = torch.randn(37, hidden, device=DEV, dtype=dtype)
    w = torch.randn(hidden, device=DEV, dtype=dtype)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    _close(ops.rms_norm(x, w, 1e-6), ref.rms_norm(x.float(), w.float(), 1e-6), tol, 1e-2)
    r = torch.randn_like(x)
    r_ref = r.clone()
    y, r_out = ops.fused_add_rms_norm(x, r, w, 1e-6)
    y_ref, rr = ref.fused_add_rms_norm(x, r_ref, w, 1e-6)
    _close(r_out, rr, tol, 1e-2)
    _close(y, y_ref, tol * 2, 2e-2)


def test_silu_and_mul():
    x = torch.randn(19, 2 * 1408, device=DEV, dtype=torch.bfloat16)
    _close(ops.silu_and_mul(x), ref.silu_and_mul(x.float()), 2e-2, 1e-2)


@pytest.mark.parametrize("interleaved", [True, False])
def test_rope(interleaved):
    cs = ref.rope_cos_sin_cache(64, 512, 10000.0, {"type": "yarn", "factor": 40, "beta_fast": 32, "beta_slow": 1,
                                                   "mscale": 0.707, "mscale_all_dim": 0.707,
                                                   "original_max_position_embeddings": 4096}, DEV)
    q = torch.randn(9, 16, 192, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 512, (9,), device=DEV)
    expect = ref.apply_rope(q[..., 128:].float(), pos, cs, interleaved=interleaved)
    ops.rope_(q[..., 128:], pos, cs, interleaved=interleaved)
    _close(q[..., 128:], expect, 3e-2, 1e-2)


@pytest.mark.parametrize("cfg", [
    dict(E=64, k=6, scoring="softmax", renormalize=False),
    dict(E=128, k=8, scoring="softmax", renormalize=True),
    dict(E=256, k=8, scoring="sigmoid", renormalize=True, n_group=8, topk_group=4, routed_scaling_factor=2.5),
    dict(E=16, k=4, scoring="softmax", renormalize=False, n_group=4, topk_group=2),
])
def test_topk_route(cfg):
    cfg = dict(cfg)
    E, k = cfg.pop("E"), cfg.pop("k")
    logits = torch.randn(200, E, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1 if cfg["scoring"] == "sigmoid" else None
    w, ids = ops.topk_route(logits, k, bias=bias, **cfg)
    w_ref, ids_ref = ref.topk_route(logits.cpu(), k, bias=None if bias is None else bias.cpu(), **cfg)
    assert torch.equal(ids.cpu(), ids_ref)
    _close(w, w_ref, 1e-5, 1e-5)


@pytest.mark.parametrize("renorm", [True, False])
def test_topk_route_sqrtsoftplus_and_hash(renorm):
    """DeepSeek-V4 routing: sqrt(softplus) scores with a selection bias, and hash-forced experts."""
    E, k = 64, 6
    logits = torch.randn(150, E, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1
    cfg = dict(scoring="sqrtsoftplus", renormalize=renorm, routed_scaling_factor=1.5)
    w, ids = ops.topk_route(logits, k, bias=bias, **cfg)
    w_ref, ids_ref = ref.topk_route(logits.cpu(), k, bias=bias.cpu(), **cfg)
    assert torch.equal(ids.cpu(), ids_ref)
    _close(w, w_ref, 1e-5, 1e-5)
    forced = torch.randint(0, E, (150, k), device=DEV, dtype=torch.int32)
    w, ids = ops.topk_route(logits, k, forced_ids=forced, **cfg)
    w_ref, ids_ref = ref.topk_route(logits.cpu(), k, forced_ids=forced.cpu(), **cfg)
    assert torch.equal(ids.cpu(), ids_ref)
    _close(w, w_ref, 1e-5, 1e-5)


def _paged_cache(B, lens, width, bs=64, dtype=torch.bfloat16, extra_blocks=3):
    nblk_seq = [math.ceil(n / bs) for n in lens]
    total = sum(nblk_seq) + extra_blocks
    cache = torch.randn(total, bs, width, device=DEV, dtype=dtype)
    perm = torch.randperm(total - 1)[: sum(nblk_seq)] + 1
    table = torch.zeros(B, max(nblk_seq), dtype=torch.int32)
    o = 0
    for b, nb in enumerate(nblk_seq):
        table[b, :nb] = perm[o : o + nb].to(torch.int32)
        o += nb
    return cache, table.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("heads", [16, 32, 128])
@pytest.mark.parametrize("splits", [1, 0, 3])
def test_mla_decode(heads, splits):
    """MLA decode (tcgen05 kernel: 16 heads per CTA, 32 from 64 heads up) vs fp32."""
    torch.manual_seed(heads + splits)
    lens = [1, 31, 32, 33, 64, 200, 1029]
    B = len(lens)
    cache, table, seq = _paged_cache(B, lens, 576)
    q = torch.randn(B, heads, 576, device=DEV, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(192)
    out = ops.mla_decode(q, cache, table, seq, scale, 512, num_splits=splits)
    expect = ref.mla_decode(q.float(), cache.float(), table, seq, scale, 512)
    _close(out, expect, 2e-2, 2e-2)


@pytest.mark.parametrize("hq,hkv", [(32, 4), (8, 8), (16, 2)])
@pytest.mark.parametrize("splits", [1, 0])
def test_gqa_decode(hq, hkv, splits):
    torch.manual_seed(hq + hkv + splits)
    lens = [1, 30, 64, 65, 333]
    B = len(lens)
    kc, table, seq = _paged_cache(B, lens, hkv * 128)
    kc = kc.view(kc.shape[0], kc.shape[1], hkv, 128)
    vc = torch.randn_like(kc)
    q = torch.randn(B, hq, 128, device=DEV, dtype=torch.bfloat16)
    out = ops.gqa_decode(q, kc, vc, table, seq, 0.088, num_splits=splits)
    expect = ref.gqa_decode(q.float(), kc.float(), vc.float(), table, seq, 0.088)
    _close(out, expect, 2e-2, 2e-2)


def test_mla_cache_write():
    T, L, R = 11, 512, 64
    kv_a = torch.randn(T, L + R, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(L, device=DEV, dtype=torch.bfloat16)
    cs = ref.rope_cos_sin_cache(R, 256, 10000.0, None, DEV)
    pos = torch.randint(0, 256, (T,), device=DEV)
    cache = torch.zeros(4, 64, L + R, device=DEV, dtype=torch.bfloat16)
    slots = torch.randperm(256, device=DEV)[:T]
    ops.mla_cache_write(cache, kv_a, w, 1e-6, pos, cs, slots, L)
    flat = cache.view(-1, L + R)[slots]
    _close(flat[:, :L], ref.rms_norm(kv_a[:, :L].float(), w.float(), 1e-6), 3e-2, 2e-2)
    _close(flat[:, L:], ref.apply_rope(kv_a[:, None, L:].float(), pos, cs, interleaved=True)[:, 0], 3e-2, 2e-2)


@pytest.mark.parametrize("shape", [(64, 6, 8, 256, 128), (300, 6, 64, 2048, 1408), (40, 8, 16, 512, 768),
                                   (700, 2, 4, 256, 128)])
def test_moe_experts_grouped_gemm(shape):
    T, k, E, H, I = shape
    torch.manual_seed(T)
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device=DEV, dtype=torch.bfloat16) * 0.05
    w2 = torch.randn(E, H, I, device=DEV, dtype=torch.bfloat16) * 0.05
    logits = torch.randn(T, E, device=DEV)
    tw, tid = ref.topk_route(logits, k, renormalize=True)
    out = ops.moe_experts(x, w13, w2, tw, tid)
    expect = ref.moe_experts(x.float(), w13.float(), w2.float(), tw, tid)
    scale = expect.abs().max().item()
    _close(out / scale, expect / scale, 2e-2)


def test_moe_expert_parallel_slice():
    T, k, E, H, I = 50, 4, 16, 256, 128
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device=DEV, dtype=torch.bfloat16) * 0.05
    w2 = torch.randn(E, H, I, device=DEV, dtype=torch.bfloat16) * 0.05
    tw, tid = ref.topk_route(torch.randn(T, E, device=DEV), k)
    full = ref.moe_experts(x.float(), w13.float(), w2.float(), tw, tid)
    part = sum(ops.moe_experts(x, w13[o:o + 8], w2[o:o + 8], tw, tid, expert_offset=o).float() for o in (0, 8))
    _close(part, full, 3e-2, 3e-2)


def _quant_experts(w):
    qs, ss = zip(*(ref.quant_fp8_block_weight(w[e].float()) for e in range(w.shape[0])))
    q, s = torch.stack(qs), torch.stack(ss)
    deq = torch.stack([ref.dequant_block(q[e], s[e]) for e in range(w.shape[0])])
    return q, s.contiguous(), deq


@pytest.mark.parametrize("counts_list", [[3, 0, 130, 64], [1, 1, 1, 1, 1, 1, 1, 1], [200], [16, 17, 33, 5]])
@pytest.mark.parametrize("epilogue", [0, 1])
def test_grouped_gemm_w8_matches_dequantised_reference(counts_list, epilogue):
    """fp8 block-scaled weights (tiles dequantised in shared memory) vs fp32 math on the
    dequantised weights (segments of 1-200 tokens: N rounded to 16, several passes)."""
    torch.manual_seed(len(counts_list) * 10 + epilogue)
    C = _ext.ops()
    E, K, N = len(counts_list), 512, 384 if epilogue == 0 else 512
    counts = torch.tensor(counts_list, dtype=torch.int32, device=DEV)
    offsets = torch.zeros(E, dtype=torch.int32, device=DEV)
    offsets[1:] = counts.cumsum(0)[:-1]
    R = int(counts.sum())
    a = (torch.randn(R + 5, K, device=DEV) * 0.5).to(torch.bfloat16)
    w = torch.randn(E, N, K, device=DEV) * 0.05
    q, s, deq = _quant_experts(w)
    out = C.grouped_gemm_w8(a, q, s, offsets, counts, epilogue, E)
    torch.cuda.synchronize()
    for e in range(E):
        o, c = int(offsets[e]), int(counts[e])
        if c == 0:
            continue
        y = a[o : o + c].float() @ deq[e].t()
        if epilogue == 1:
            g, u = y[:, : N // 2], y[:, N // 2 :]
            y = g * torch.sigmoid(g) * u
        got = out[o : o + c].float()
        sc = y.abs().max().item() + 1e-6
        _close(got / sc, y / sc, 2e-2)


def test_moe_experts_fp8_weights():
    T, k, E, H, I = 96, 6, 16, 512, 256
    torch.manual_seed(5)
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    q13, s13, d13 = _quant_experts(torch.randn(E, 2 * I, H, device=DEV) * 0.05)
    q2, s2, d2 = _quant_experts(torch.randn(E, H, I, device=DEV) * 0.05)
    tw, tid = ref.topk_route(torch.randn(T, E, device=DEV), k, renormalize=True)
    out = ops.moe_experts(x, q13, q2, tw, tid, w13_scale=s13, w2_scale=s2)
    expect = ref.moe_experts(x.float(), d13, d2, tw, tid)
    scale = expect.abs().max().item()
    _close(out / scale, expect / scale, 2e-2)


@pytest.mark.parametrize("heads,bs", [(16, 64), (32, 16)])
@pytest.mark.parametrize("splits", [1, 0, 3])
def test_mla_decode_sparse(heads, bs, splits):
    """Gather kernel over kept positions: -1 entries, positions out of order, rows of any block size."""
    torch.manual_seed(7 * heads + splits)
    lens = [1, 40, 97, 300, 1029]
    B, K = len(lens), 96
    cache, table, seq = _paged_cache(B, lens, 576, bs=bs)
    keep = torch.full((B, K), -1, dtype=torch.int32)
    for b, n in enumerate(lens):
        pick = torch.randperm(n)[: min(n, K - 5)]
        keep[b, torch.randperm(K)[: len(pick)]] = pick.to(torch.int32)
    keep = keep.to(DEV)
    q = torch.randn(B, heads, 576, device=DEV, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(192)
    out = _ext.ops().mla_decode_sparse(q, cache, table, seq, keep, scale, splits)
    expect = ref.mla_decode_sparse(q.float(), cache.float(), table, keep, scale, 512)
    _close(out, expect, 2e-2, 2e-2)


def test_mla_decode_sparse_routing(monkeypatch):
    """The op takes the kernel under the switch and agrees with the gather + GEMM form."""
    torch.manual_seed(3)
    lens = [50, 130]
    cache, table, seq = _paged_cache(2, lens, 576)
    keep = torch.stack([torch.randperm(130)[:64] % n for n in lens]).to(torch.int64).to(DEV)
    q = torch.randn(2, 16, 576, device=DEV, dtype=torch.bfloat16)
    monkeypatch.setenv("AFD_SPARSE_MLA_KERNEL", "0")
    base = ops.mla_decode_sparse(q, cache, table, seq, keep, 0.1, 512)
    monkeypatch.setenv("AFD_SPARSE_MLA_KERNEL", "1")
    assert ops.sparse_kernel_enabled()
    got = ops.mla_decode_sparse(q, cache, table, seq, keep, 0.1, 512)
    _close(got, base, 2e-2, 2e-2)


def _segments(counts_list):
    counts = torch.tensor(counts_list, dtype=torch.int32, device=DEV)
    offsets = torch.zeros(len(counts_list), dtype=torch.int32, device=DEV)
    offsets[1:] = counts.cumsum(0)[:-1]
    return counts, offsets, int(counts.sum())


def _swiglu_ref(a, w13, w2=None):
    y = a.float() @ w13.float().t()
    i = y.shape[1] // 2
    h = torch.nn.functional.silu(y[:, :i]) * y[:, i:]
    return h if w2 is None else h.to(torch.bfloat16).float() @ w2.float().t()


@pytest.mark.parametrize("counts_list", [[24, 0, 31, 256, 1, 64, 65, 130], [300, 3], [7] * 20])
@pytest.mark.parametrize("epilogue", [0, 1])
def test_grouped_gemm_activation_ring(counts_list, epilogue):
    """Passes of 1-4 activation slots (and several passes for > 256 rows) vs fp32 per segment."""
    torch.manual_seed(sum(counts_list) + epilogue)
    C = _ext.ops()
    counts, offsets, R = _segments(counts_list)
    E, K, N = len(counts_list), 256, 384 if epilogue == 0 else 256
    a = (torch.randn(R + 3, K, device=DEV) * 0.5).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device=DEV) * 0.05).to(torch.bfloat16)
    out = C.grouped_gemm(a, w, offsets, counts, epilogue)
    torch.cuda.synchronize()
    for e in range(E):
        o, c = int(offsets[e]), int(counts[e])
        if c == 0:
            continue
        y = _swiglu_ref(a[o : o + c], w[e]) if epilogue == 1 else a[o : o + c].float() @ w[e].float().t()
        sc = y.abs().max().item() + 1e-6
        _close(out[o : o + c] / sc, y / sc, 2e-2)


@pytest.mark.parametrize("counts_list,H,I", [([24, 31, 0, 17, 256, 256], 512, 256), ([300, 5, 70], 256, 128),
                                             ([3] * 66, 2048, 1408)])
def test_moe_ffn_two_phase(counts_list, H, I):
    """gate_up -> SwiGLU -> down in one launch vs fp32, twice in a row; the counters end at zero."""
    from afd_plugin_b200.ops.moe import moe_sync_buffer

    torch.manual_seed(len(counts_list) + H)
    C = _ext.ops()
    counts, offsets, R = _segments(counts_list)
    E = len(counts_list)
    w13 = (torch.randn(E, 2 * I, H, device=DEV) * 0.04).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device=DEV) * 0.04).to(torch.bfloat16)
    sync = moe_sync_buffer(torch.device(DEV), E)
    for rep in range(2):
        a = (torch.randn(R + 2, H, device=DEV) * 0.5).to(torch.bfloat16)
        y = C.moe_ffn(a, w13, w2, offsets, counts, sync, max(counts_list))
        torch.cuda.synchronize()
        assert int(sync.abs().sum()) == 0, "moe_ffn must leave its counters at zero"
        for e in range(E):
            o, c = int(offsets[e]), int(counts[e])
            if c == 0:
                continue
            want = _swiglu_ref(a[o : o + c], w13[e], w2[e])
            sc = want.abs().max().item() + 1e-6
            _close(y[o : o + c] / sc, want / sc, 3e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [102400, 1000, 37])
def test_argmax_rows(dtype, n):
    torch.manual_seed(n)
    x = torch.randn(67, n, device=DEV).to(dtype)
    x[3, :] = 0  # ties: the lowest index wins, as torch.argmax
    x[5, n // 2] = x[5].max() + 1
    x[5, n - 1] = x[5, n // 2]
    got = _ext.ops().argmax_rows(x)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu().long(), torch.argmax(x.float(), dim=-1).cpu())


@pytest.mark.parametrize("T,N,K", [(256, 3712, 2048), (43, 2048, 2048), (1, 128, 64), (300, 102400 // 8, 2048)])
def test_tc_gemm_dense(T, N, K):
    torch.manual_seed(T + N)
    x = (torch.randn(T, K, device=DEV) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.03).to(torch.bfloat16)
    y = _ext.ops().tc_gemm(x, w, 0)
    want = x.float() @ w.float().t()
    sc = want.abs().max().item()
    _close(y / sc, want / sc, 2e-2)


def test_tc_gemm_strided_rows_and_swiglu():
    torch.manual_seed(3)
    big = (torch.randn(77, 3712, device=DEV) * 0.5).to(torch.bfloat16)
    x = big[:, :2048]  # rows 3712 elements apart
    w = (torch.randn(512, 2048, device=DEV) * 0.03).to(torch.bfloat16)
    y = _ext.ops().tc_gemm(x, w, 1)
    want = _swiglu_ref(x, w)
    sc = want.abs().max().item()
    _close(y / sc, want / sc, 2e-2)


def test_tc_gemm_per_head_batched():
    """MLA absorption shapes: q_nope heads read in place from the projection output, written token-major."""
    torch.manual_seed(4)
    T, nh = 37, 16
    y = (torch.randn(T, 3712, device=DEV) * 0.5).to(torch.bfloat16)
    q_nope = y[:, : nh * 192].view(T, nh, 192)[..., :128].transpose(0, 1)  # [16, T, 128], strided
    w_uk_t = (torch.randn(nh, 512, 128, device=DEV) * 0.05).to(torch.bfloat16)
    out = _ext.ops().tc_gemm(q_nope, w_uk_t)  # [T, 16 * 512]
    want = torch.einsum("htk,hnk->thn", q_nope.float(), w_uk_t.float()).reshape(T, nh * 512)
    sc = want.abs().max().item()
    _close(out / sc, want / sc, 2e-2)
    o_lat = (torch.randn(nh, T, 512, device=DEV) * 0.5).to(torch.bfloat16)  # head-major, contiguous
    w_uv = (torch.randn(nh, 128, 512, device=DEV) * 0.05).to(torch.bfloat16)
    o = _ext.ops().tc_gemm(o_lat, w_uv)  # [T, 16 * 128]
    want = torch.einsum("htk,hnk->thn", o_lat.float(), w_uv.float()).reshape(T, nh * 128)
    sc = want.abs().max().item()
    _close(o / sc, want / sc, 2e-2)


@pytest.mark.parametrize("T,N,K,n_valid,f32", [(256, 3712, 2048, 0, False), (43, 2048, 2048, 0, False),
                                              (256, 128, 2048, 64, True), (7, 128, 512, 100, False)])
def test_tc_gemm_split_k(T, N, K, n_valid, f32):
    """Few output tiles: K split over the SMs with fp32 partial sums; the workspace is left zero."""
    from afd_plugin_b200.ops.moe import gemm_workspace

    torch.manual_seed(T * 3 + N)
    ws, ctr = gemm_workspace(torch.device(DEV))
    x = (torch.randn(T, K, device=DEV) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.03).to(torch.bfloat16)
    for _ in range(2):
        y = _ext.ops().tc_gemm(x, w, 0, n_valid, f32, ws, ctr)
        torch.cuda.synchronize()
        assert int(ctr.abs().sum()) == 0 and float(ws.abs().sum()) == 0.0
    want = x.float() @ w.float().t()
    if n_valid:
        want = want[:, :n_valid]
    assert y.dtype == (torch.float32 if f32 else torch.bfloat16) and tuple(y.shape) == tuple(want.shape)
    sc = want.abs().max().item()
    _close(y / sc, want / sc, 2e-2)


def test_tc_gemm_split_k_per_head():
    from afd_plugin_b200.ops.moe import gemm_workspace

    torch.manual_seed(9)
    ws, ctr = gemm_workspace(torch.device(DEV))
    o_lat = (torch.randn(16, 64, 512, device=DEV) * 0.5).to(torch.bfloat16)
    w_uv = (torch.randn(16, 128, 512, device=DEV) * 0.05).to(torch.bfloat16)
    o = _ext.ops().tc_gemm(o_lat, w_uv, 0, 0, False, ws, ctr)
    want = torch.einsum("htk,hnk->thn", o_lat.float(), w_uv.float()).reshape(64, 16 * 128)
    sc = want.abs().max().item()
    _close(o / sc, want / sc, 2e-2)
    torch.cuda.synchronize()
    assert int(ctr.abs().sum()) == 0 and float(ws.abs().sum()) == 0.0


def test_mla_decode_split_merge_repeats():
    """Split partials merged inside the launch: the arrival counters reset, so
    back-to-back launches (64 requests, one wave of splits) all match fp32."""
    torch.manual_seed(11)
    lens = torch.randint(300, 1100, (64,)).tolist()
    cache, table, seq = _paged_cache(64, lens, 576)
    scale = 1 / math.sqrt(192)
    for rep in range(3):
        q = torch.randn(64, 16, 576, device=DEV, dtype=torch.bfloat16)
        out = ops.mla_decode(q, cache, table, seq, scale, 512)
        expect = ref.mla_decode(q.float(), cache.float(), table, seq, scale, 512)
        _close(out, expect, 2e-2, 2e-2)


def test_mla_cache_write_rotates_query():
    """The cache-write launch also applies the query's interleaved RoPE in place (strided q_pe view)."""
    T, H, L, R = 13, 16, 512, 64
    torch.manual_seed(5)
    kv_a = torch.randn(T, L + R, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(L, device=DEV, dtype=torch.bfloat16)
    cs = ref.rope_cos_sin_cache(R, 256, 10000.0, None, DEV)
    pos = torch.randint(0, 256, (T,), device=DEV)
    cache = torch.zeros(4, 64, L + R, device=DEV, dtype=torch.bfloat16)
    slots = torch.randperm(256, device=DEV)[:T]
    q = torch.randn(T, H, 192, device=DEV, dtype=torch.bfloat16)
    q_pe = q[..., 128:]
    expect_q = ref.apply_rope(q_pe.float(), pos, cs, interleaved=True)
    nope_before = q[..., :128].clone()
    ops.mla_cache_write(cache, kv_a, w, 1e-6, pos, cs, slots, L, q_pe=q_pe)
    _close(q[..., 128:], expect_q, 3e-2, 2e-2)
    assert torch.equal(q[..., :128], nope_before)
    flat = cache.view(-1, L + R)[slots]
    _close(flat[:, L:], ref.apply_rope(kv_a[:, None, L:].float(), pos, cs, interleaved=True)[:, 0], 3e-2, 2e-2)


@pytest.mark.parametrize("shape", ["32,2", "32,4", "64,2"])
def test_mla_decode_tc_shapes_16_heads(shape):
    """The tcgen05 MLA kernel's 16-heads-per-CTA shapes (selected only through
    AFD_MLA_TC_SHAPE, read once per process, hence the child process) vs fp32."""
    import os
    import subprocess
    import sys

    code = (
        "import math, torch\n"
        "from afd_plugin_b200 import ops\n"
        "from afd_plugin_b200.ops import reference as ref\n"
        "torch.manual_seed(0)\n"
        "lens=[1,33,64,200,1029]\n"
        "bs=64\n"
        "nb=[math.ceil(n/bs) for n in lens]\n"
        "cache=torch.randn(sum(nb)+2,bs,576,device='cuda',dtype=torch.bfloat16)\n"
        "table=torch.zeros(len(lens),max(nb),dtype=torch.int32)\n"
        "o=1\n"
        "for b,k in enumerate(nb):\n"
        "    table[b,:k]=torch.arange(o,o+k,dtype=torch.int32); o+=k\n"
        "table=table.cuda(); seq=torch.tensor(lens,dtype=torch.int32,device='cuda')\n"
        "for heads in (16, 32):\n"
        "    for splits in (1, 0, 3):\n"
        "        q=torch.randn(len(lens),heads,576,device='cuda',dtype=torch.bfloat16)\n"
        "        out=ops.mla_decode(q,cache,table,seq,0.07,512,num_splits=splits).float()\n"
        "        exp=ref.mla_decode(q.float(),cache.float(),table,seq,0.07,512)\n"
        "        err=((out-exp).abs().max()/(exp.abs().max()+1e-6)).item()\n"
        "        assert err < 2e-2, (heads, splits, err)\n"
        "print('ok')\n"
    )
    env = dict(os.environ, AFD_MLA_TC_SHAPE=shape)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


@pytest.mark.skipif(os.environ.get("AFD_RUN_UNVERIFIED_KERNELS") != "1",
                    reason="the work-balanced MLA kernel has not run on a GPU yet; AFD_RUN_UNVERIFIED_KERNELS=1 runs it")
def test_mla_decode_balanced_vs_fp32():
    """The work-balanced MLA decode kernel (AFD_MLA_BALANCED=1, read once per process, hence the child
    process) vs fp32: mixed lengths, one request over many CTAs, more CTAs than tiles, 16 and 128 heads,
    and repeated launches (the per-request arrival counters must be left at zero)."""
    import subprocess
    import sys

    code = (
        "import math, torch\n"
        "from afd_plugin_b200 import ops\n"
        "from afd_plugin_b200.ops import reference as ref\n"
        "torch.manual_seed(0)\n"
        "bs=64\n"
        "for lens, heads in (([1,33,64,200,1029], 16), ([20000], 16), ([1034]*300, 16), ([5,700,64,1], 128),\n"
        "                    ([2,3], 16)):\n"
        "    nb=[math.ceil(n/bs) for n in lens]\n"
        "    cache=torch.randn(sum(nb)+2,bs,576,device='cuda',dtype=torch.bfloat16)\n"
        "    table=torch.zeros(len(lens),max(nb),dtype=torch.int32)\n"
        "    o=1\n"
        "    for b,k in enumerate(nb):\n"
        "        table[b,:k]=torch.arange(o,o+k,dtype=torch.int32); o+=k\n"
        "    table=table.cuda(); seq=torch.tensor(lens,dtype=torch.int32,device='cuda')\n"
        "    for rep in range(3):\n"
        "        q=torch.randn(len(lens),heads,576,device='cuda',dtype=torch.bfloat16)\n"
        "        out=ops.mla_decode(q,cache,table,seq,0.07,512).float()\n"
        "        exp=ref.mla_decode(q.float(),cache.float(),table,seq,0.07,512)\n"
        "        err=((out-exp).abs().max()/(exp.abs().max()+1e-6)).item()\n"
        "        assert err < 2e-2, (len(lens), heads, rep, err)\n"
        "assert torch.ops.afd_b200.read_status(0) == 0\n"
        "print('ok')\n"
    )
    env = dict(os.environ, AFD_MLA_BALANCED="1", AFD_MLA_KERNEL="mma")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


def test_gate_sigmoid_rows():
    """Qwen3.5 shared-expert gate: sigmoid(x . w) per row, written into each chunk's routing weights."""
    torch.manual_seed(4)
    R, H, copies, span = 37, 2048, 3, 40
    x = torch.randn(R, H, device=DEV).to(torch.bfloat16)
    w = (torch.randn(H, device=DEV) * 0.02).to(torch.bfloat16)
    out = torch.full((copies * span,), -1.0, device=DEV)
    _ext.ops().gate_sigmoid_rows(x, w, out, copies, span)
    expect = torch.sigmoid(x.float() @ w.float())
    for c in range(copies):
        _close(out[c * span : c * span + R], expect, 1e-4, 1e-4)
        assert bool((out[c * span + R : (c + 1) * span] == -1.0).all())


@pytest.mark.parametrize("nq,nkv,d,norm", [(32, 4, 128, True), (8, 8, 128, False), (4, 2, 64, True), (6, 2, 32, True)])
def test_gqa_prologue_matches_unfused(nq, nkv, d, norm):
    """q / k RMSNorm + NeoX RoPE + k / v cache write in one kernel vs the
    separate norm, rope and cache-write ops (fp32 reference math)."""
    torch.manual_seed(nq + d)
    T, bs = 9, 16
    qkv_full = torch.randn(T, (nq + 2 * nkv) * d + 8, device=DEV).to(torch.bfloat16)
    qkv = qkv_full[:, 8:]  # strided rows
    qw = (1 + 0.1 * torch.randn(d, device=DEV)).to(torch.bfloat16) if norm else None
    kw = (1 + 0.1 * torch.randn(d, device=DEV)).to(torch.bfloat16) if norm else None
    cs = ref.rope_cos_sin_cache(d, 512, 10000.0, None, DEV)
    pos = torch.randint(0, 512, (T,), device=DEV)
    slots = torch.randperm(4 * bs, device=DEV)[:T]
    kc = torch.zeros(4, bs, nkv, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = ops.gqa_prologue(qkv, nq, nkv, d, qw, kw, 1e-6, pos, cs, kc, vc, slots)
    qf, kf, vf = qkv.float().split([nq * d, nkv * d, nkv * d], dim=-1)
    qf, kf = qf.reshape(T, nq, d), kf.reshape(T, nkv, d)
    if norm:
        qf = ref.rms_norm(qf, qw.float(), 1e-6)
        kf = ref.rms_norm(kf, kw.float(), 1e-6)
    qf = ref.apply_rope(qf, pos, cs, interleaved=False)
    kf = ref.apply_rope(kf, pos, cs, interleaved=False)
    _close(q.float(), qf, 3e-2, 2e-2)
    _close(kc.view(-1, nkv, d)[slots].float(), kf, 3e-2, 2e-2)
    assert torch.equal(vc.view(-1, nkv, d)[slots], qkv[:, (nq + nkv) * d :].reshape(T, nkv, d))
