"""vLLM version handling.

This package runs on its own engine and needs no vLLM.  vLLM matters in two
places: the plugin hook may publish the ``AFD<Arch>`` names into vLLM's
``ModelRegistry`` (``register_afd``), and the bench's reference arm runs the
reference plugin, which supports exactly one vLLM release
(``afd_plugin/compat/vllm.py:12`` pins 0.26.0 and refuses others,
``assert_vllm_version_supported``).  This module answers both questions
from the installed distribution's metadata without importing vLLM.
"""

from __future__ import annotations

import re
import warnings
from importlib.metadata import PackageNotFoundError, version

# The release the reference plugin is written against (its engine-core and
# forward-context patches target that release's internals).
REFERENCE_VLLM_VERSION = "0.26.0"
# ``ModelRegistry.register_model(name, "module:Class")`` with lazy class
# strings, which the alias publishing uses.
MIN_REGISTRY_VLLM_VERSION = "0.6.0"


def release(v: str) -> tuple[int, int, int]:
    """``major.minor.patch`` of a version string (local / dev suffixes ignored)."""
    m = re.match(r"^\s*v?(\d+)\.(\d+)(?:\.(\d+))?", v)
    if m is None:
        raise ValueError(f"cannot parse a vLLM version from {v!r}")
    return int(m.group(1)), int(m.group(2)), int(m.group(3) or 0)


def installed_vllm_version() -> str | None:
    """The installed vLLM distribution's version, or None (read from metadata; vLLM is not imported)."""
    try:
        return version("vllm")
    except PackageNotFoundError:
        return None


def reference_vllm_mismatch(installed: str | None = None) -> str | None:
    """Why the reference plugin cannot run on ``installed`` (default: this environment's vLLM), or None."""
    installed = installed_vllm_version() if installed is None else installed
    if installed is None:
        return "vLLM is not installed (the reference plugin runs inside vLLM)"
    if release(installed) != release(REFERENCE_VLLM_VERSION):
        return (f"the reference plugin supports exactly vLLM {REFERENCE_VLLM_VERSION}; "
                f"vLLM {installed} is installed")
    return None


def can_publish_aliases(installed: str | None = None, *, strict: bool = False) -> bool:
    """Whether ``register_afd`` can publish its names into this vLLM's ``ModelRegistry``.

    False without vLLM or below ``MIN_REGISTRY_VLLM_VERSION``; ``strict``
    raises instead of warning for a too-old release.
    """
    installed = installed_vllm_version() if installed is None else installed
    if installed is None:
        return False
    if release(installed) >= release(MIN_REGISTRY_VLLM_VERSION):
        return True
    msg = (f"vLLM {installed} predates lazy ModelRegistry entries ({MIN_REGISTRY_VLLM_VERSION}+); "
           "the AFD aliases are not published")
    if strict:
        raise RuntimeError(msg)
    warnings.warn(msg, RuntimeWarning, stacklevel=2)
    return False


__all__ = ["MIN_REGISTRY_VLLM_VERSION", "REFERENCE_VLLM_VERSION", "can_publish_aliases", "installed_vllm_version",
           "reference_vllm_mismatch", "release"]
