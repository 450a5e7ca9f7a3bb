"""Tensor-parallel all-reduce over NVLink peer memory (one kernel, no library call).

:class:`PeerAllReduce` sums a ``[rows, H]`` bf16 tensor in place over a
process group whose ranks share one node: every rank pushes its rows into a
slot of every rank's symmetric heap with plain stores, releases an
epoch-tagged flag per CTA, waits (bounded) for its peers' flags and adds the
slots locally in fp32 (``ops/csrc/tp_allreduce.cu``).  The epoch lives on the
device, so a call replays from a CUDA graph.  It serves the row-parallel
``o_proj`` of tensor-parallel attention; tensors larger than its slots go to
``torch.distributed.all_reduce``.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from afd_plugin_b200.parallel.symm_heap import HeapLayout, SymmetricHeap

MAX_CTAS = 1024


class PeerAllReduce:
    """Collective constructor over ``group`` (every member passes the same sizes)."""

    def __init__(self, group, *, max_rows: int, hidden: int, device: int | None = None,
                 timeout_ms: int | None = None):
        from afd_plugin_b200.ops._ext import ops

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.cuda.current_device() if device is None else device
        self.slot_elems = int(max_rows) * int(hidden)
        layout = HeapLayout()
        layout.add("slots", (2, self.world, self.slot_elems), torch.bfloat16)
        layout.add("flags", (MAX_CTAS, self.world), torch.int64)
        self.heap = SymmetricHeap(layout, group=group, device=self.device)
        self.heap.view("flags").zero_()
        dev = torch.device("cuda", self.device)
        ranks = list(range(self.world))
        self.slot_ptrs = self.heap.ptr_table(ranks, "slots")
        self.flag_ptrs = self.heap.ptr_table(ranks, "flags")
        self.local_slots = self.heap.view("slots")
        self.local_flags = self.heap.view("flags")
        self.epoch = torch.ones(1, dtype=torch.int64, device=dev)  # flags start at 0
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        ms = timeout_ms if timeout_ms is not None else int(os.environ.get("AFD_B200_WAIT_TIMEOUT_MS", "10000"))
        self.timeout_ns = int(ms) * 1_000_000
        self._op = ops().tp_allreduce_
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals

    def fits(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous()
                and x.numel() <= self.slot_elems and x.shape[1] % 8 == 0 and x.data_ptr() % 16 == 0)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """Sum ``x`` over the group in place (``torch.distributed`` for tensors that do not fit)."""
        if self.world == 1:
            return x
        if not self.fits(x):
            dist.all_reduce(x, group=self.group)
            return x
        self._op(x, self.slot_ptrs, self.flag_ptrs, self.local_slots, self.local_flags, self.epoch, self.done,
                 self.rank, self.world, self.slot_elems, MAX_CTAS, self.timeout_ns)
        return x

    def close(self) -> None:
        self.heap.close()


__all__ = ["MAX_CTAS", "PeerAllReduce"]
