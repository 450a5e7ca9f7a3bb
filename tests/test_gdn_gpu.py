"""Gated DeltaNet kernels (causal conv + recurrent delta rule) vs the fp32 reference."""

import pytest
import torch

from afd_plugin_b200.ops import _ext
from afd_plugin_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    C = _ext.ops()
    C.reset_status(0)
    yield
    torch.cuda.synchronize()
    assert C.read_status(0) == 0


def _cu(lens):
    return torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("K", [4, 2])
def test_gdn_conv_prefill_then_decode(K):
    torch.manual_seed(K)
    C = _ext.ops()
    ch, lens, slots_n = 96, [5, 1, 17], 6
    w = (torch.randn(ch, K, device=DEV) * 0.5).to(torch.bfloat16)
    state = torch.randn(slots_n, ch, K - 1, device=DEV).to(torch.bfloat16)
    slots = torch.tensor([4, 0, 2], dtype=torch.int32, device=DEV)
    reset = torch.tensor([1, 0, 1], dtype=torch.int32, device=DEV)
    T = sum(lens)
    wide = torch.randn(T, ch + 40, device=DEV).to(torch.bfloat16)  # strided rows: channels are a prefix
    x = wide[:, :ch]
    init = state.clone()
    y = C.gdn_conv(x, w, state, _cu(lens), slots, reset)
    torch.cuda.synchronize()
    t0 = 0
    for i, n in enumerate(lens):
        st0 = None if reset[i] else init[slots[i]].float()
        y_ref, st_ref = ref.causal_conv1d(x[t0 : t0 + n], w, st0)
        torch.testing.assert_close(y[t0 : t0 + n].float(), y_ref, atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(state[slots[i]].float(), st_ref, atol=1e-2, rtol=1e-2)
        t0 += n
    # untouched slots keep their contents
    for sl in (1, 3, 5):
        assert torch.equal(state[sl], init[sl])


@pytest.mark.parametrize("nk,nv,dk", [(2, 4, 32), (1, 2, 64), (2, 4, 128)])
def test_gdn_recurrent_prefill_then_decode(nk, nv, dk):
    torch.manual_seed(nk * 100 + dk)
    C = _ext.ops()
    dv = dk
    lens = [7, 1, 3]
    slots_n = 5
    T = sum(lens)
    width = 2 * nk * dk + nv * dv
    qkv = torch.randn(T, width, device=DEV).to(torch.bfloat16)
    z = torch.randn(T, nv * dv, device=DEV).to(torch.bfloat16)
    ab = torch.randn(T, 2 * nv, device=DEV).to(torch.bfloat16)
    b, a = ab[:, :nv], ab[:, nv:]
    A_log = torch.randn(nv, device=DEV) * 0.5
    dt_bias = torch.randn(nv, device=DEV) * 0.5
    norm_w = (1 + 0.1 * torch.randn(dv, device=DEV)).to(torch.bfloat16)
    state = torch.randn(slots_n, nv, dk, dv, device=DEV) * 0.1
    slots = torch.tensor([3, 1, 0], dtype=torch.int32, device=DEV)
    reset = torch.tensor([1, 0, 0], dtype=torch.int32, device=DEV)
    init = state.clone()
    out = C.gdn_recurrent(qkv, z, a, b, A_log, dt_bias, norm_w, 1e-6, state, _cu(lens), slots, reset, nk)
    torch.cuda.synchronize()
    r = nv // nk
    t0 = 0
    for i, n in enumerate(lens):
        sl = slots[i]
        seg = qkv[t0 : t0 + n].float()
        q = seg[:, : nk * dk].view(n, nk, dk).repeat_interleave(r, dim=1)
        k = seg[:, nk * dk : 2 * nk * dk].view(n, nk, dk).repeat_interleave(r, dim=1)
        v = seg[:, 2 * nk * dk :].view(n, nv, dv)
        g, beta = ref.gdn_gates(a[t0 : t0 + n], b[t0 : t0 + n], A_log, dt_bias)
        st0 = None if reset[i] else init[sl]
        o, st = ref.gated_delta_rule(q, k, v, g, beta, st0)
        want = ref.rms_norm_gated(o, z[t0 : t0 + n].view(n, nv, dv), norm_w, 1e-6).reshape(n, nv * dv)
        torch.testing.assert_close(out[t0 : t0 + n].float(), want, atol=3e-2, rtol=3e-2)
        torch.testing.assert_close(state[sl], st, atol=2e-3, rtol=2e-3)
        t0 += n
    for sl in (2, 4):
        assert torch.equal(state[sl], init[sl])
