"""Role profiler: environment parsing and a recorded trace on CPU."""

import os

import pytest
import torch

from afd_plugin_b200.utils.profiler import RoleProfiler, profiler_settings


def test_defaults_and_parsing(monkeypatch):
    for k in list(os.environ):
        if k.startswith("AFD_GPU_") or k == "VLLM_TORCH_PROFILER_DIR":
            monkeypatch.delenv(k, raising=False)
    s = profiler_settings("ffn")
    assert not s.enabled and s.wait == 2500 and s.active == 10 and s.trace_dir == "./profiler_logs/ffn"
    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_ENABLE", "yes")
    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_WAIT", "3")
    monkeypatch.setenv("VLLM_TORCH_PROFILER_DIR", "/tmp/x")
    s = profiler_settings("attention")
    assert s.enabled and s.wait == 3 and s.trace_dir == "/tmp/x"
    monkeypatch.setenv("AFD_GPU_FFN_PROFILER_ENABLE", "perhaps")
    with pytest.raises(ValueError):
        profiler_settings("ffn")
    with pytest.raises(ValueError):
        profiler_settings("router")


def test_trace_written(tmp_path, monkeypatch):
    monkeypatch.setenv("AFD_GPU_FFN_PROFILER_ENABLE", "1")
    monkeypatch.setenv("AFD_GPU_FFN_PROFILER_WAIT", "1")
    monkeypatch.setenv("AFD_GPU_FFN_PROFILER_ACTIVE", "2")
    monkeypatch.setenv("AFD_GPU_FFN_PROFILER_DIR", str(tmp_path))
    p = RoleProfiler("ffn")
    assert p.enabled
    for _ in range(5):
        torch.randn(64, 64) @ torch.randn(64, 64)
        p.step()
    p.close()
    assert any(f.name.endswith(".json") or ".pt.trace" in f.name for f in tmp_path.iterdir())


def test_engine_steps_are_named_in_the_attention_trace(tmp_path, monkeypatch):
    from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
    from afd_plugin_b200.models import build_model, get_preset
    from afd_plugin_b200.runtime.engine import LLMEngine

    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_ENABLE", "1")
    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_WAIT", "0")
    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_WARMUP", "0")
    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_ACTIVE", "4")
    monkeypatch.setenv("AFD_GPU_ATTENTION_PROFILER_DIR", str(tmp_path))
    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64), max_num_seqs=2)
    eng = LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=64))
    eng.generate([[1, 2, 3]], 4)
    eng.close()
    text = "".join(f.read_text(errors="replace") for f in tmp_path.iterdir() if f.is_file())
    assert "afd_prefill_step" in text and "afd_decode_step" in text
