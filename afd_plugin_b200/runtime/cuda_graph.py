"""When the AFD roles run a decode step as a CUDA graph, and which graph (torch-free).

A decode step of this framework is one CUDA graph per role and step shape:

* Attention ranks capture one graph per padded batch size
  (:func:`pad_to_capture_size`).
* FFN ranks capture one graph per *key*.  The fused connector keeps token
  counts in device memory and sizes every buffer by capacity, so its key is
  the stage set and the capacity (:func:`capacity_graph_key`): one capture
  serves any routing and any batch up to the capacity.  The NCCL connector
  moves tensors whose shapes are the token counts, so its key is what each
  FFN rank receives per stage (:func:`count_graph_key`).  That key keeps the
  layout ``((stage, per-FFN-rank counts), ...)`` of the reference's FFN runner
  (``afd_plugin/v1/worker/cuda_graph.py:104-133``), so the two stacks capture
  one graph per distinct traffic pattern alike.

Only ``FULL_DECODE_ONLY`` is accepted (the reference states the same rule,
``afd_plugin/v1/worker/cuda_graph.py:42-85``): prefill runs eagerly.  DBO
with graphs needs exactly two ubatches, because the captured step
interleaves two ubatch generators.  The run mode of an FFN step follows the
control payload's flags (:func:`pick_run_mode`).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from enum import Enum
from typing import Any

from afd_plugin_b200.runtime.ffn_metadata import aggregate_ffn_token_counts

GRAPH_MODE = "FULL_DECODE_ONLY"


class RunMode(str, Enum):
    EAGER = "eager"  # run the step's kernels directly
    WARMUP = "warmup"  # eager, to initialise lazily created state before a capture
    CAPTURE = "capture"  # record the step into a new graph
    REPLAY = "replay"  # launch the recorded graph


@dataclass(frozen=True, slots=True)
class GraphSettings:
    """What the engine configuration allows for one role."""

    enabled: bool  # graphs at all (False under enforce_eager)
    mode: str | None  # the configured graph mode's name
    attention_graphs: bool  # this role captures Attention decode steps
    ffn_graphs: bool  # this role keeps a cache of FFN step graphs
    two_ubatches: bool = False  # the captured step interleaves two DBO ubatches


def graph_mode_name(config: Any) -> str | None:
    """Name of ``config.compilation_config.cudagraph_mode`` (an enum, its name or its str form)."""
    raw = getattr(getattr(config, "compilation_config", None), "cudagraph_mode", None)
    if raw is None:
        return None
    name = getattr(raw, "name", None)
    if not isinstance(name, str):
        name = str(raw)
    return name.split(".")[-1] or None


def graph_settings(config: Any, *, role: str | None = None) -> GraphSettings:
    """Checks the graph configuration of ``role`` ("attention", "ffn" or None for both).

    Raises ``RuntimeError`` for a mode other than ``FULL_DECODE_ONLY`` or for
    DBO with a ubatch count other than two, unless ``enforce_eager`` is set.
    """
    mode = graph_mode_name(config)
    if getattr(config.model_config, "enforce_eager", False):
        return GraphSettings(False, mode, False, False)
    who = f"the {role} role" if role else "AFD"
    if mode != GRAPH_MODE:
        raise RuntimeError(f"CUDA graphs for {who} run only as {GRAPH_MODE} (got {mode!r}); "
                           "set enforce_eager to run without graphs.")
    par = getattr(config, "parallel_config", None)
    ubatched = bool(getattr(par, "use_ubatching", False))
    if ubatched:
        n = getattr(par, "num_ubatches", None)
        if int(n or 0) != 2:
            raise RuntimeError(f"a captured DBO step for {who} interleaves exactly two ubatches "
                               f"({GRAPH_MODE}); got num_ubatches={n!r}.")
    return GraphSettings(
        enabled=True,
        mode=mode,
        attention_graphs=role in (None, "attention"),
        ffn_graphs=role in (None, "ffn"),
        two_ubatches=ubatched,
    )


def _stage_counts(meta: Any) -> tuple[int, ...]:
    """Per-Attention-rank (or per-DP-rank) token counts carried by a stage's metadata."""
    raw = getattr(meta, "num_tokens_across_dp_cpu", meta)
    if raw is None:
        return ()
    if hasattr(raw, "tolist"):
        raw = raw.tolist()
    if isinstance(raw, (int, float)):
        return (int(raw),)
    return tuple(int(v) for v in raw)


def count_graph_key(stage_meta: Mapping[int, Any], *, attention_size: int | None = None,
                    ffn_size: int | None = None) -> tuple:
    """FFN graph key of the NCCL connector: ``((stage, counts), ...)`` in stage order.

    With both sizes given, the counts are what each FFN rank receives (its
    Attention peers' counts, an empty peer sending one placeholder row;
    :func:`aggregate_ffn_token_counts`); otherwise they are the raw counts.
    """
    key = []
    fold = bool(attention_size) and bool(ffn_size)
    for stage in sorted(stage_meta):
        counts = _stage_counts(stage_meta[stage])
        if fold:
            counts = aggregate_ffn_token_counts(counts, attention_size=int(attention_size), ffn_size=int(ffn_size))
        key.append((int(stage), counts))
    return tuple(key)


def capacity_graph_key(stages: tuple[int, ...], capacity: int) -> tuple:
    """FFN graph key of the fused connector: the stage set and the per-rank token capacity."""
    return ("capacity", tuple(sorted(int(s) for s in stages)), int(capacity))


def pick_run_mode(*, warmup: bool, capturing: bool, replaying: bool, graphs_on: bool, have_graph: bool) -> RunMode:
    """Run mode of an FFN step from the control payload's flags.

    A warm-up or capture request wins over replay; a replay request without
    a recorded graph (or with graphs off) runs eagerly.
    """
    if warmup:
        return RunMode.WARMUP
    if capturing:
        return RunMode.CAPTURE
    return RunMode.REPLAY if (replaying and graphs_on and have_graph) else RunMode.EAGER


def pad_to_capture_size(num_tokens: int, capture_sizes: list[int] | tuple[int, ...]) -> int | None:
    """Smallest capture size >= ``num_tokens`` (``None`` -> run eagerly)."""
    fits = [s for s in capture_sizes if s >= num_tokens]
    return min(fits) if fits else None


__all__ = [
    "GRAPH_MODE",
    "GraphSettings",
    "RunMode",
    "capacity_graph_key",
    "count_graph_key",
    "graph_mode_name",
    "graph_settings",
    "pad_to_capture_size",
    "pick_run_mode",
]
