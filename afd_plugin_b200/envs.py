"""Environment switches read by the framework.

``AFD_FORCE_BALANCED_TOPK_IDS`` mirrors ``afd_plugin/envs.py:9-14`` of the
reference; the ``AFD_B200_*`` names are this framework's own.
"""

from __future__ import annotations

import os

AFD_FORCE_BALANCED_TOPK_IDS = "AFD_FORCE_BALANCED_TOPK_IDS"
# Bound (milliseconds) on every device-side wait for a peer flag.
AFD_B200_WAIT_TIMEOUT_MS = "AFD_B200_WAIT_TIMEOUT_MS"
# Debug builds of the CUDA kernels check every index and record violations.
AFD_B200_KERNEL_DEBUG = "AFD_B200_KERNEL_DEBUG"
# Seconds without a peer heartbeat before a worker reports the peer dead (unset: no heartbeat).
AFD_HEARTBEAT_TIMEOUT_S = "AFD_HEARTBEAT_TIMEOUT_S"
ENV_TRUE_VALUES = frozenset({"1", "true", "yes", "on"})


def _flag(name: str) -> bool:
    return os.environ.get(name, "").strip().lower() in ENV_TRUE_VALUES


def force_balanced_topk_ids_enabled() -> bool:
    return _flag(AFD_FORCE_BALANCED_TOPK_IDS)


def kernel_debug_enabled() -> bool:
    return _flag(AFD_B200_KERNEL_DEBUG)


def wait_timeout_ms(default: int = 2000) -> int:
    raw = os.environ.get(AFD_B200_WAIT_TIMEOUT_MS, "").strip()
    if not raw:
        return default
    value = int(raw)
    if value <= 0:
        raise ValueError(f"{AFD_B200_WAIT_TIMEOUT_MS} must be positive, got {value}")
    return value


__all__ = [
    "AFD_B200_KERNEL_DEBUG",
    "AFD_B200_WAIT_TIMEOUT_MS",
    "AFD_FORCE_BALANCED_TOPK_IDS",
    "force_balanced_topk_ids_enabled",
    "kernel_debug_enabled",
    "wait_timeout_ms",
]


def heartbeat_timeout_s() -> float | None:
    raw = os.environ.get(AFD_HEARTBEAT_TIMEOUT_S, "").strip()
    if not raw:
        return None
    value = float(raw)
    if value <= 0:
        raise ValueError(f"{AFD_HEARTBEAT_TIMEOUT_S} must be positive, got {value}")
    return value
