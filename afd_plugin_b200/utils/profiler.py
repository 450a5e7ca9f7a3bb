"""Per-role torch.profiler traces for AFD serving (opt-in through the environment).

Environment (``<P>`` is ``AFD_GPU_ATTENTION_PROFILER`` or ``AFD_GPU_FFN_PROFILER``),
the same knobs as the reference (``afd_plugin/compat/profiler.py:19-60``):

* ``<P>_ENABLE``      1/true to record (default off)
* ``<P>_WAIT``        steps skipped per cycle before warm-up (default 2500)
* ``<P>_WARMUP``      warm-up steps (default 1)
* ``<P>_ACTIVE``      recorded steps (default 10)
* ``<P>_REPEAT``      cycles (default 1)
* ``<P>_SKIP_FIRST``  steps skipped once at the start (default 0)
* ``<P>_DIR``         TensorBoard trace directory (falls back to
  ``VLLM_TORCH_PROFILER_DIR``, then ``./profiler_logs/{attn,ffn}``)

A step is one engine step on the Attention side and one served control
payload on the FFN side.  Device timings inside a profiled run are for
inspection only, never for benchmark numbers.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass

log = logging.getLogger(__name__)

_PREFIX = {"attention": "AFD_GPU_ATTENTION_PROFILER", "ffn": "AFD_GPU_FFN_PROFILER"}
_DIR = {"attention": "./profiler_logs/attn", "ffn": "./profiler_logs/ffn"}


@dataclass(frozen=True)
class ProfilerSettings:
    enabled: bool
    wait: int
    warmup: int
    active: int
    repeat: int
    skip_first: int
    trace_dir: str


def _flag(name: str, default: bool) -> bool:
    raw = os.getenv(name)
    if raw is None:
        return default
    v = raw.strip().lower()
    if v in ("1", "true", "yes", "on"):
        return True
    if v in ("0", "false", "no", "off"):
        return False
    raise ValueError(f"{name} must be a boolean, got {raw!r}")


def _count(name: str, default: int) -> int:
    raw = os.getenv(name)
    if raw is None:
        return default
    try:
        return int(raw)
    except ValueError as exc:
        raise ValueError(f"{name} must be an integer, got {raw!r}") from exc


def profiler_settings(role: str) -> ProfilerSettings:
    if role not in _PREFIX:
        raise ValueError(f"profiler role must be 'attention' or 'ffn', got {role!r}")
    p = _PREFIX[role]
    return ProfilerSettings(
        enabled=_flag(f"{p}_ENABLE", False),
        wait=_count(f"{p}_WAIT", 2500),
        warmup=_count(f"{p}_WARMUP", 1),
        active=_count(f"{p}_ACTIVE", 10),
        repeat=_count(f"{p}_REPEAT", 1),
        skip_first=_count(f"{p}_SKIP_FIRST", 0),
        trace_dir=os.getenv(f"{p}_DIR") or os.getenv("VLLM_TORCH_PROFILER_DIR") or _DIR[role],
    )


class RoleProfiler:
    """Step-scheduled torch.profiler; a no-op when the role's ENABLE is off."""

    def __init__(self, role: str):
        self.settings = profiler_settings(role)
        self._prof = None
        if not self.settings.enabled:
            return
        import torch

        s = self.settings
        log.info("AFD %s profiler on; traces go to %s", role, s.trace_dir)
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self._prof = torch.profiler.profile(
            activities=acts,
            schedule=torch.profiler.schedule(wait=s.wait, warmup=s.warmup, active=s.active, repeat=s.repeat,
                                             skip_first=s.skip_first),
            on_trace_ready=torch.profiler.tensorboard_trace_handler(s.trace_dir),
            record_shapes=True,
        )
        self._prof.start()

    @property
    def enabled(self) -> bool:
        return self._prof is not None

    def step(self) -> None:
        if self._prof is not None:
            self._prof.step()

    def close(self) -> None:
        if self._prof is not None:
            self._prof.stop()
            self._prof = None


__all__ = ["ProfilerSettings", "RoleProfiler", "profiler_settings"]
