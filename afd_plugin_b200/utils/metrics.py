"""Per-step serving metrics: rolling summary and optional JSONL stream.

``AFD_METRICS_JSONL=<path>`` appends one JSON object per engine step
(phase, batch, generated tokens, step milliseconds, host<->device bytes, HBM
bytes the step must move).  ``StepMetrics.summary()`` gives tokens/s, p50 /
p90 step time, the decode steps' HBM bytes per second and their fraction of
the measured HBM bandwidth (``utils/roofline.py``), and, with
``AFD_PHASE_TIMING=1``, the latest step's per-phase device microseconds
(``utils/phase_timer.py``).  Step times are host wall-clock around a step that
ends with the device->host read of its tokens, so they include the device
work; benchmark numbers come from CUDA events in ``bench.py`` instead.
"""

from __future__ import annotations

import json
import os
import time
from collections import deque


class StepMetrics:
    def __init__(self, path: str | None = None, *, keep: int = 100_000):
        self.path = path if path is not None else os.environ.get("AFD_METRICS_JSONL") or None
        self.keep = keep
        # the most recent ``keep`` decode steps: (ms, tokens)
        self._window: deque[tuple[float, int, int]] = deque(maxlen=keep)
        self.phases: dict = {}  # latest decode step's phase timing (when enabled)
        self.decode_tokens = 0
        self.steps = 0
        self._fh = open(self.path, "a", buffering=1) if self.path else None  # noqa: SIM115

    def record(self, *, phase: str, batch: int, tokens: int, ms: float, h2d_bytes: int = 0,
               d2h_bytes: int = 0, hbm_bytes: int = 0) -> None:
        self.steps += 1
        if phase == "decode":
            self.decode_tokens += tokens
            self._window.append((ms, tokens, hbm_bytes))
        if self._fh is not None:
            self._fh.write(json.dumps({"step": self.steps, "phase": phase, "batch": batch, "tokens": tokens,
                                       "ms": round(ms, 4), "h2d_bytes": h2d_bytes, "d2h_bytes": d2h_bytes,
                                       "hbm_bytes": hbm_bytes, "t": round(time.time(), 6)}) + "\n")

    @property
    def decode_ms(self) -> list[float]:
        return [m for m, _, _ in self._window]

    def summary(self) -> dict:
        """Totals since start; rates and percentiles over the most recent ``keep`` decode steps."""
        ms = sorted(self.decode_ms)
        if not ms:
            return {"steps": self.steps, "decode_steps": 0}
        pick = lambda q: ms[min(len(ms) - 1, int(q * (len(ms) - 1) + 0.5))]  # noqa: E731
        total_s = sum(ms) / 1e3
        window_tokens = sum(t for _, t, _ in self._window)
        out = {"steps": self.steps, "decode_steps": len(ms), "decode_tokens": self.decode_tokens,
               "decode_tok_per_s": round(window_tokens / total_s, 2) if total_s > 0 else 0.0,
               "p50_step_ms": round(pick(0.5), 4), "p90_step_ms": round(pick(0.9), 4)}
        hbm = sum(b for _, _, b in self._window)
        if hbm and total_s > 0:
            from afd_plugin_b200.utils.roofline import hbm_peak_gbs

            peak, kind = hbm_peak_gbs()
            gbs = hbm / total_s / 1e9
            out["hbm_bytes_per_step"] = int(hbm / len(ms))
            out["hbm_GBps"] = round(gbs, 1)
            out[f"frac_of_{kind}_hbm"] = round(gbs / peak, 3)
        if self.phases:
            out["phases_us"] = self.phases
        return out

    def close(self) -> None:
        if self._fh is not None:
            self._fh.close()
            self._fh = None


__all__ = ["StepMetrics"]
