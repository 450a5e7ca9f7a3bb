"""AFD across two GPUs (one process per GPU): NCCL baseline and fused B200 connector.

The NCCL connector runs the same FFN ops as the colocated model, so its tokens
must match exactly.  The fused connector normalises, routes and sums in its own
kernels (different bf16 rounding points), so it is held to near-agreement.
"""

import pytest
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.launcher import LocalAFDSpec, launch_local

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
PRESET = "tiny-dsv2-mla512"


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _prompts(n, length, vocab=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g).tolist()


def _colocated(prompts, max_tokens, preset=PRESET):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.bfloat16, enforce_eager=True, max_model_len=128), max_num_seqs=8)
    m = build_model(arch, role="colocated", dtype=torch.bfloat16, device="cuda", seed=0, max_positions=128)
    return LLMEngine(ec, m).generate(prompts, max_tokens)


def _run(afd, prompts, max_tokens, preset=PRESET, logits=False, **kw):
    spec = LocalAFDSpec(preset=preset, afd=afd, prompts=prompts, max_tokens=max_tokens, dtype="bfloat16",
                        backend="nccl", record_logits_steps=2 if logits else 0, **kw)
    res = launch_local(spec, join_timeout_s=240)
    errs = {r: v for r, v in res.items() if "error" in v}
    assert not errs, errs
    outs = []
    for r in sorted(res):
        outs += res[r].get("outputs", [])
    if logits:
        steps = [v["logits"] for v in res.values() if v.get("role") == "attention"]
        return outs, [torch.from_numpy(a) for a in steps[0]]
    return outs


def _colocated_logits(prompts, steps=2, preset=PRESET):
    """Logits of the colocated model's first engine steps (the prefill, then the first decode step)."""
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.bfloat16, enforce_eager=True, max_model_len=128), max_num_seqs=8)
    m = build_model(arch, role="colocated", dtype=torch.bfloat16, device="cuda", seed=0, max_positions=128)
    eng = LLMEngine(ec, m)
    for p in prompts:
        eng.add_request(p, 6)
    out = []
    for _ in range(steps):
        eng.step()
        out.append(eng.runner.last_logits[: len(prompts)].float().cpu())
    return out


def _rel_max_diff(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def _agreement(a, b):
    flat_a = [t for o in a for t in o]
    flat_b = [t for o in b for t in o]
    return sum(x == y for x, y in zip(flat_a, flat_b)) / max(1, len(flat_a))


def test_nccl_connector_1a1f_exact():
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated(prompts, 6)
    outs = _run({"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts, 6)
    assert outs == ref


def test_nccl_connector_1a1f_graphs_exact():
    """Stream-ordered NCCL sends / receives captured into both roles' decode graphs."""
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated(prompts, 6)
    outs = _run({"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts, 6, enforce_eager=False, capture_sizes=[4])
    assert outs == ref


@pytest.mark.parametrize("eager,dbo", [(True, False), (False, False), (False, True)])
def test_fused_connector_1a1f(eager, dbo):
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated(prompts, 6)
    afd = {"num_attention_ranks": 1, "num_ffn_ranks": 1, "connector": "B200FusedAFDConnector",
           "connector_extra_config": {"max_tokens_per_rank": 128, "wait_timeout_ms": 20000}}
    outs = _run(afd, prompts, 6, enforce_eager=eager, use_ubatching=dbo, capture_sizes=[4])
    assert [o[0] for o in outs] == [o[0] for o in ref]
    assert _agreement(outs, ref) >= 0.75


def test_fused_connector_qwen3_5_1a1f():
    """Hybrid Gated DeltaNet model through the fused connector (gated shared expert on the FFN side)."""
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated(prompts, 6, preset="tiny-qwen3.5")
    afd = {"num_attention_ranks": 1, "num_ffn_ranks": 1, "connector": "B200FusedAFDConnector",
           "connector_extra_config": {"max_tokens_per_rank": 128, "wait_timeout_ms": 20000}}
    outs = _run(afd, prompts, 6, preset="tiny-qwen3.5", enforce_eager=False, capture_sizes=[4])
    assert [o[0] for o in outs] == [o[0] for o in ref]
    assert _agreement(outs, ref) >= 0.75


def test_fused_connector_dsv4_1a1f():
    """mHC on the Attention side (pre-normalised dispatch) and hash routing in the router kernel."""
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated(prompts, 6, preset="tiny-dsv4")
    afd = {"num_attention_ranks": 1, "num_ffn_ranks": 1, "connector": "B200FusedAFDConnector",
           "connector_extra_config": {"max_tokens_per_rank": 128, "wait_timeout_ms": 20000}}
    outs = _run(afd, prompts, 6, preset="tiny-dsv4", enforce_eager=False, capture_sizes=[4])
    assert [o[0] for o in outs] == [o[0] for o in ref]
    assert _agreement(outs, ref) >= 0.75


def test_fused_connector_fp8_rows_1a1f():
    """e4m3 rows (1 x 128 scales) across NVLink: held to near-agreement with the bf16 colocated model."""
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated(prompts, 6)
    afd = {"num_attention_ranks": 1, "num_ffn_ranks": 1, "connector": "B200FusedAFDConnector",
           "connector_extra_config": {"max_tokens_per_rank": 128, "wait_timeout_ms": 20000, "fp8_dispatch": True}}
    outs = _run(afd, prompts, 6, enforce_eager=False, capture_sizes=[4])
    assert _agreement(outs, ref) >= 0.5


def test_nccl_connector_1a1f_logits_match():
    """Prefill and first decode step logits through the NCCL connector equal the
    colocated model's (the same ops on the same bf16 values)."""
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated_logits(prompts)
    _, got = _run({"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts, 6, logits=True)
    assert len(got) == 2
    for step, (g, r) in enumerate(zip(got, ref)):
        assert g.shape == r.shape
        assert _rel_max_diff(g, r) <= 1e-3, (step, _rel_max_diff(g, r))


@pytest.mark.parametrize("eager", [True, False])
def test_fused_connector_1a1f_logits_close(eager):
    """Prefill and first decode step logits through the fused connector stay within
    bf16 tolerance of the colocated model's: the kernels normalise, route and
    sum with other bf16 rounding points, so the bound is 3 % of the largest
    logit (max abs difference), and the arg-max token matches."""
    _need(2)
    prompts = _prompts(4, 16)
    ref = _colocated_logits(prompts)
    afd = {"num_attention_ranks": 1, "num_ffn_ranks": 1, "connector": "B200FusedAFDConnector",
           "connector_extra_config": {"max_tokens_per_rank": 128, "wait_timeout_ms": 20000}}
    _, got = _run(afd, prompts, 6, logits=True, enforce_eager=eager, capture_sizes=[4])
    assert len(got) == 2
    for step, (g, r) in enumerate(zip(got, ref)):
        assert g.shape == r.shape
        d = _rel_max_diff(g, r)
        assert d <= 3e-2, (step, d)
        assert torch.equal(g.argmax(-1), r.argmax(-1)), step
