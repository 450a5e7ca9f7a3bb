"""CUDA-graph policy for AFD roles (importable without torch).

Rules match ``afd_plugin/v1/worker/cuda_graph.py:42-150``: only
``FULL_DECODE_ONLY`` is accepted; ubatching (DBO) with graphs needs exactly
two ubatches; the FFN graph key is ``((stage, per-FFN-rank token counts), ...)``
and the FFN run mode comes from the control payload flags.

The fused B200 connector keeps token counts on the device, so its FFN graphs
are keyed by the stage set and the padded capacity only
(:func:`make_capacity_graph_key`): one capture serves any routing.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from enum import Enum
from typing import Any

FULL_DECODE_ONLY = "FULL_DECODE_ONLY"
_SUPPORTED = frozenset({FULL_DECODE_ONLY})


class AFDGraphRunMode(str, Enum):
    EAGER = "eager"
    WARMUP = "warmup"
    CAPTURE = "capture"
    REPLAY = "replay"


@dataclass(frozen=True, slots=True)
class AFDCUDAGraphPolicy:
    enabled: bool
    mode_name: str | None
    allow_attention_full_decode_only: bool
    enable_ffn_graph_cache: bool
    allow_cuda_graph_with_ubatching: bool = False


def cudagraph_mode_name(config: Any) -> str | None:
    mode = getattr(getattr(config, "compilation_config", None), "cudagraph_mode", None)
    if mode is None:
        return None
    name = getattr(mode, "name", None)
    if isinstance(name, str):
        return name
    text = str(mode)
    return (text.rsplit(".", 1)[-1] if "." in text else text) or None


def validate_cuda_graph_mode(config: Any, *, role: str | None = None) -> AFDCUDAGraphPolicy:
    eager = bool(getattr(config.model_config, "enforce_eager", False))
    mode = cudagraph_mode_name(config)
    if eager:
        return AFDCUDAGraphPolicy(False, mode, False, False)
    if mode not in _SUPPORTED:
        suffix = f" for {role}" if role else ""
        raise RuntimeError(f"AFD only supports CUDA graph mode {FULL_DECODE_ONLY}{suffix}; got {mode!r}.")
    par = getattr(config, "parallel_config", None)
    ubatching = bool(getattr(par, "use_ubatching", False))
    n_ub = getattr(par, "num_ubatches", None)
    ub_ok = ubatching and int(n_ub or 0) == 2
    if ubatching and not ub_ok:
        raise RuntimeError(
            f"AFD CUDA graph support currently supports ubatching only for {FULL_DECODE_ONLY} with exactly two "
            f"ubatches; got num_ubatches={n_ub!r}."
        )
    return AFDCUDAGraphPolicy(
        enabled=True,
        mode_name=mode,
        allow_attention_full_decode_only=role in (None, "attention"),
        enable_ffn_graph_cache=role in (None, "ffn"),
        allow_cuda_graph_with_ubatching=ub_ok,
    )


def _values(values: Any) -> tuple[int, ...]:
    tolist = getattr(values, "tolist", None)
    if callable(tolist):
        values = tolist()
    elif hasattr(values, "item"):
        values = [values.item()]
    try:
        return tuple(int(v) for v in values)
    except TypeError:
        return (int(values),)


def _aggregated_key_applies(attention_size: int | None, ffn_size: int | None) -> bool:
    return (
        attention_size is not None
        and ffn_size is not None
        and int(attention_size) >= int(ffn_size)
        and int(attention_size) % int(ffn_size) == 0
    )


def _aggregate(values: tuple[int, ...], *, attention_size: int, ffn_size: int, fallback: int) -> tuple[int, ...]:
    expanded = values
    if len(values) < attention_size and values and attention_size % len(values) == 0:
        tp = attention_size // len(values)
        expanded = tuple(values[i // tp] for i in range(attention_size))
    if len(expanded) < attention_size:
        return tuple(max(1, int(fallback)) for _ in range(ffn_size))
    g = attention_size // ffn_size
    return tuple(max(1, sum(expanded[i * g : (i + 1) * g])) for i in range(ffn_size))


def make_ffn_graph_key(
    dp_metadata_list: Mapping[int, object],
    *,
    attention_size: int | None = None,
    ffn_size: int | None = None,
    fallback: int = 1,
) -> tuple:
    parts = []
    agg = _aggregated_key_applies(attention_size, ffn_size)
    for stage, meta in sorted(dp_metadata_list.items()):
        raw = getattr(meta, "num_tokens_across_dp_cpu", None)
        if raw is None:
            vals = tuple(max(1, int(fallback)) for _ in range(int(ffn_size))) if agg else (repr(meta),)
        else:
            vals = _values(raw)
            if agg:
                vals = _aggregate(vals, attention_size=int(attention_size), ffn_size=int(ffn_size),
                                  fallback=int(fallback))
        parts.append((int(stage), vals))
    return tuple(parts)


def make_capacity_graph_key(stages: tuple[int, ...], capacity: int) -> tuple:
    """Graph key of the fused connector: counts live on the device."""
    return ("capacity", tuple(sorted(int(s) for s in stages)), int(capacity))


def graph_run_mode(
    *, is_warmup: bool, is_graph_capturing: bool, is_graph_replaying: bool, graph_enabled: bool, graph_exists: bool
) -> AFDGraphRunMode:
    if is_warmup:
        return AFDGraphRunMode.WARMUP
    if is_graph_capturing:
        return AFDGraphRunMode.CAPTURE
    if is_graph_replaying and graph_enabled and graph_exists:
        return AFDGraphRunMode.REPLAY
    return AFDGraphRunMode.EAGER


def pad_to_capture_size(num_tokens: int, capture_sizes: list[int] | tuple[int, ...]) -> int | None:
    """Smallest capture size >= ``num_tokens`` (``None`` -> run eagerly)."""
    fits = [s for s in capture_sizes if s >= num_tokens]
    return min(fits) if fits else None


__all__ = [
    "AFDCUDAGraphPolicy",
    "AFDGraphRunMode",
    "FULL_DECODE_ONLY",
    "cudagraph_mode_name",
    "graph_run_mode",
    "make_capacity_graph_key",
    "make_ffn_graph_key",
    "pad_to_capture_size",
    "validate_cuda_graph_mode",
]
