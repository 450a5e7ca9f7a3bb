"""vLLM version handling: release parsing, the reference plugin's exact pin, alias publishing."""

import pytest

from afd_plugin_b200 import compat


def test_release_parsing():
    assert compat.release("0.26.0") == (0, 26, 0)
    assert compat.release("0.22.1+cu128") == (0, 22, 1)
    assert compat.release("v1.2") == (1, 2, 0)
    assert compat.release("0.26.0rc1.dev5") == (0, 26, 0)
    with pytest.raises(ValueError):
        compat.release("nightly")


def test_reference_pin_is_exact():
    assert compat.reference_vllm_mismatch("0.26.0") is None
    assert compat.reference_vllm_mismatch("0.26.0+cu129") is None
    msg = compat.reference_vllm_mismatch("0.22.0")
    assert "exactly vLLM 0.26.0" in msg and "0.22.0" in msg
    assert "0.27.1" in compat.reference_vllm_mismatch("0.27.1")


def test_alias_publishing_needs_a_recent_vllm():
    assert compat.can_publish_aliases("0.22.0")
    with pytest.warns(RuntimeWarning):
        assert not compat.can_publish_aliases("0.5.4")
    with pytest.raises(RuntimeError):
        compat.can_publish_aliases("0.5.4", strict=True)


def test_installed_version_is_read_from_metadata(monkeypatch):
    from importlib.metadata import PackageNotFoundError

    def missing(name):
        raise PackageNotFoundError(name)

    monkeypatch.setattr(compat, "version", missing)
    assert compat.installed_vllm_version() is None
    assert "not installed" in compat.reference_vllm_mismatch()
    assert not compat.can_publish_aliases()
    monkeypatch.setattr(compat, "version", lambda name: "0.26.0")
    assert compat.reference_vllm_mismatch() is None
