"""Package surface and the ``vllm.general_plugins`` entry point (CPU only).

Mirrors the reference's package test (``tests/unit/package/test_package.py``):
the entry point named in the build script resolves to a callable, the
registration is idempotent, every alias resolves to a wrapper class, and a
registry stand-in records what would be published into vLLM.
"""

from __future__ import annotations

import importlib
import re
import sys
import types
from pathlib import Path

import pytest

import afd_plugin_b200 as pkg

ROOT = Path(__file__).resolve().parents[1]


def _entry_point() -> str:
    text = (ROOT / "setup.py").read_text()
    m = re.search(r'"vllm\.general_plugins":\s*\["afd = ([\w.]+:\w+)"\]', text)
    assert m, "setup.py must declare the vllm.general_plugins entry point"
    return m.group(1)


def test_version_and_exports():
    assert re.fullmatch(r"\d+\.\d+\.\d+", pkg.__version__)
    for name in pkg.__all__:
        assert getattr(pkg, name) is not None
    with pytest.raises(AttributeError):
        pkg.NoSuchThing  # noqa: B018


def test_entry_point_resolves_to_register_afd():
    mod, fn = _entry_point().split(":")
    assert getattr(importlib.import_module(mod), fn) is pkg.register_afd


@pytest.fixture
def fresh_registration(monkeypatch):
    from afd_plugin_b200.models import MODEL_REGISTRY

    monkeypatch.setattr(pkg, "_REGISTERED", False)
    saved = dict(MODEL_REGISTRY)
    yield MODEL_REGISTRY
    MODEL_REGISTRY.clear()
    MODEL_REGISTRY.update(saved)


def test_register_without_vllm_is_idempotent(monkeypatch, fresh_registration):
    monkeypatch.setitem(sys.modules, "vllm", None)  # import of vllm fails
    first = pkg.register_afd()
    second = pkg.register_afd()
    assert first == second == pkg.MODEL_ALIASES
    from afd_plugin_b200.models import model as model_mod

    for arch, alias in pkg.MODEL_ALIASES.items():
        assert fresh_registration[alias] is fresh_registration[arch]
        assert isinstance(getattr(model_mod, pkg._class_name(alias)), type)


class _FakeRegistry:
    def __init__(self, supported):
        self.supported = list(supported)
        self.registered: dict[str, str] = {}

    def get_supported_archs(self):
        return self.supported + list(self.registered)

    def register_model(self, name, target):
        self.registered[name] = target


def test_vllm_registry_untouched_by_default(monkeypatch, fresh_registration):
    reg = _FakeRegistry(["DeepseekV2ForCausalLM"])
    monkeypatch.setitem(sys.modules, "vllm", types.SimpleNamespace(ModelRegistry=reg))
    monkeypatch.delenv("AFD_PUBLISH_VLLM_ALIASES", raising=False)
    assert pkg.register_afd() == pkg.MODEL_ALIASES
    assert reg.registered == {}


def test_register_publishes_lazy_targets_into_vllm(monkeypatch, fresh_registration):
    monkeypatch.setenv("AFD_PUBLISH_VLLM_ALIASES", "1")
    reg = _FakeRegistry(["DeepseekV2ForCausalLM", "AFDQwen3MoeForCausalLM"])
    monkeypatch.setitem(sys.modules, "vllm", types.SimpleNamespace(ModelRegistry=reg))
    pkg.register_afd()
    # an alias vLLM already knows is left alone
    assert "AFDQwen3MoeForCausalLM" not in reg.registered
    expected = {a for a in pkg.MODEL_ALIASES.values()} - {"AFDQwen3MoeForCausalLM"}
    assert set(reg.registered) == expected
    for alias, target in reg.registered.items():
        mod, cls = target.split(":")
        assert isinstance(getattr(importlib.import_module(mod), cls), type), alias
    assert reg.registered["AFDDeepseekV32ForCausalLM"].endswith(":AFDDeepseekV3ForCausalLM")
    # second call publishes nothing new
    n = len(reg.registered)
    pkg.register_afd()
    assert len(reg.registered) == n


def test_registry_failure_is_not_fatal(monkeypatch, fresh_registration):
    monkeypatch.setenv("AFD_PUBLISH_VLLM_ALIASES", "1")

    class Broken:
        def get_supported_archs(self):
            raise RuntimeError("registry unavailable")

    monkeypatch.setitem(sys.modules, "vllm", types.SimpleNamespace(ModelRegistry=Broken()))
    assert pkg.register_afd() == pkg.MODEL_ALIASES


def test_force_spawn_env(monkeypatch, fresh_registration):
    import multiprocessing

    calls = []
    monkeypatch.setattr(multiprocessing, "set_start_method", lambda m, force=False: calls.append((m, force)))
    monkeypatch.setitem(sys.modules, "vllm", None)
    monkeypatch.setenv("AFD_FORCE_SPAWN_MULTIPROCESSING", "1")
    monkeypatch.delenv("VLLM_WORKER_MULTIPROC_METHOD", raising=False)
    pkg.register_afd()
    import os

    assert os.environ["VLLM_WORKER_MULTIPROC_METHOD"] == "spawn"
    assert calls == [("spawn", False)]


def test_graft_entry_exposes_build_and_smoke():
    spec = importlib.util.spec_from_file_location("_graft_entry", ROOT / "__graft_entry__.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert callable(mod.build) and callable(mod.smoke)


def test_umbrella_cli_dispatches(capsys):
    from afd_plugin_b200.__main__ import COMMANDS, main

    assert main(["--help"]) == 0 and "serve" in capsys.readouterr().out
    assert main(["nope"]) == 2
    for module, fn in COMMANDS.values():
        assert callable(getattr(importlib.import_module(module), fn))
    with pytest.raises(SystemExit) as e:
        main(["serve", "--help"])
    assert e.value.code == 0
    assert "console_scripts" in (ROOT / "setup.py").read_text()
