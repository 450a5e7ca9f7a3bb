"""Count this package's kernel launches in one call (profiler, never timed)."""

from __future__ import annotations

import torch


def count_afd_kernels(fn) -> int:
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "afd::" in e.name)


__all__ = ["count_afd_kernels"]
