"""Bounded device waits: a flag nothing sets must time out with a status, not hang."""

import pytest
import torch

from afd_plugin_b200.ops import _ext

pytestmark = pytest.mark.gpu


def test_wait_times_out_and_context_survives():
    C = _ext.ops()
    C.reset_status(0)
    flag = torch.zeros(4, dtype=torch.int64, device="cuda")
    epoch = torch.ones(1, dtype=torch.int64, device="cuda")
    C.afd_wait(flag, 2, epoch, 3, 50_000_000)  # wants 3 arrivals, none come; 50 ms budget
    torch.cuda.synchronize()
    assert C.read_status(0) == 1
    C.reset_status(0)
    # the context is still usable
    x = torch.randn(8, device="cuda")
    assert torch.isfinite((x * 2).sum()).item()
    # a satisfied wait passes without touching the status
    flag[2] = 3
    C.afd_wait(flag, 2, epoch, 3, 50_000_000)
    torch.cuda.synchronize()
    assert C.read_status(0) == 0
