"""Per-role phase timing of a decode step on the device.

A :class:`PhaseTimer` places a one-thread kernel that stores the device's
global nanosecond clock at each named point of a step (``mark``).  The marks
are captured into the step's CUDA graph like every other kernel, so each
replay rewrites the same slots and the buffer holds the latest step.
:meth:`PhaseTimer.summary` turns consecutive marks into phase durations:
each phase is named by the mark that ends it and averaged over the layers.

Attention ranks mark ``attn`` (end of the layer's attention), ``dispatch``
(dispatch kernels issued and finished), ``ffn_wait`` (the FFN ranks' rows
arrived) and ``combine``.  FFN ranks mark ``arrive_wait`` (every Attention
rank's rows arrived), ``expand``, ``experts`` (grouped GEMMs) and
``combine_send``.  A phase ending in ``wait`` is time spent waiting on the
peer role; the rest is this rank's own work.  The stamp kernels serialise the
stream where they sit (no programmatic early launch across them), so enabling
timing costs a few microseconds per mark; it is off unless asked for
(``AFD_PHASE_TIMING=1`` or ``bench.py --phases``).
"""

from __future__ import annotations

import os
from collections import OrderedDict, defaultdict

import torch


def phase_timing_requested() -> bool:
    return os.environ.get("AFD_PHASE_TIMING", "") in ("1", "true", "on")


class PhaseTimer:
    def __init__(self, device, *, enabled: bool | None = None, max_marks: int = 8192):
        self.enabled = phase_timing_requested() if enabled is None else bool(enabled)
        self.device = device
        self.buf = torch.zeros(max_marks, dtype=torch.int64, device=device) if self.enabled else None
        self.names: list[str] = []
        self._pos = 0
        self._ops = None
        if self.enabled:
            from afd_plugin_b200.ops._ext import ops

            self._ops = ops()  # loads the extension (the stamp kernel lives there)

    def begin_step(self) -> None:
        """Starts the step's mark sequence (the first mark is the step's start)."""
        if not self.enabled:
            return
        self._pos = 0
        self.mark("start")

    def mark(self, name: str) -> None:
        if not self.enabled:
            return
        if self._pos >= self.buf.numel():
            return
        if self._pos < len(self.names):
            self.names[self._pos] = name
        else:
            self.names.append(name)
        self._ops.afd_stamp(self.buf, self._pos)
        self._pos += 1

    def summary(self) -> dict:
        """Phase -> {"us_per_layer", "us_per_step", "count"} for the last executed step."""
        if not self.enabled or self._pos < 2:
            return {}
        t = self.buf[: self._pos].cpu().tolist()
        per = defaultdict(list)
        for i in range(1, self._pos):
            per[self.names[i]].append((t[i] - t[i - 1]) / 1e3)
        out = OrderedDict()
        for name in self.names[1 : self._pos]:
            if name in out:
                continue
            vals = per[name]
            out[name] = {"us_per_layer": round(sum(vals) / len(vals), 2), "us_per_step": round(sum(vals), 1),
                         "count": len(vals)}
        out["step_us"] = round((t[self._pos - 1] - t[0]) / 1e3, 1)
        return out


class _NullTimer:
    enabled = False

    def begin_step(self) -> None:
        pass

    def mark(self, name: str) -> None:
        pass

    def summary(self) -> dict:
        return {}


NULL_TIMER = _NullTimer()

__all__ = ["NULL_TIMER", "PhaseTimer", "phase_timing_requested"]
