"""Per-step metrics stream and summary from a CPU engine run."""

import json

import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.utils.metrics import StepMetrics


def test_engine_writes_jsonl(tmp_path, monkeypatch):
    path = tmp_path / "m.jsonl"
    monkeypatch.setenv("AFD_METRICS_JSONL", str(path))
    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64), max_num_seqs=4)
    eng = LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64))
    eng.generate([[1, 2, 3], [4, 5, 6, 7]], 5)
    eng.close()
    rows = [json.loads(x) for x in path.read_text().splitlines()]
    assert rows[0]["phase"] == "prefill" and rows[0]["batch"] == 2
    assert [r["phase"] for r in rows[1:]] == ["decode"] * 4 and all(r["ms"] > 0 for r in rows)
    s = eng.metrics.summary()
    assert s["decode_steps"] == 4 and s["decode_tokens"] == 8 and s["p90_step_ms"] >= s["p50_step_ms"] > 0


def test_summary_percentiles():
    m = StepMetrics(path="")
    for ms in [1.0, 2.0, 3.0, 4.0, 100.0]:
        m.record(phase="decode", batch=10, tokens=10, ms=ms)
    s = m.summary()
    assert s["p50_step_ms"] == 3.0 and s["p90_step_ms"] == 100.0 and s["decode_tokens"] == 50


def test_decode_steps_report_hbm_bytes_and_roofline(tmp_path, monkeypatch):
    from afd_plugin_b200.utils.roofline import kv_bytes_per_step, weight_bytes_per_step

    path = tmp_path / "m.jsonl"
    monkeypatch.setenv("AFD_METRICS_JSONL", str(path))
    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64), max_num_seqs=4)
    model = build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64)
    eng = LLMEngine(ec, model)
    eng.generate([[1, 2, 3], [4, 5, 6, 7]], 3)
    eng.close()
    rows = [json.loads(x) for x in path.read_text().splitlines()]
    wb = weight_bytes_per_step(model)
    # embedding rows are gathered, not streamed: the table is not counted
    assert wb == sum(p.numel() * 4 for n, p in model.named_parameters() if "embed_tokens" not in n)
    first = rows[1]
    assert first["phase"] == "decode"
    # the first decode step reads contexts of 4 and 5 positions in every layer
    assert first["hbm_bytes"] == wb + kv_bytes_per_step(arch, 4 + 5, elem_bytes=4)
    s = eng.metrics.summary()
    assert s["hbm_bytes_per_step"] > wb and s["hbm_GBps"] > 0
    assert any(k.startswith("frac_of_") for k in s)


def test_roofline_peak_source():
    from afd_plugin_b200.utils.roofline import hbm_peak_gbs

    gbs, kind = hbm_peak_gbs()
    assert gbs > 1000 and kind in ("measured", "fallback")
