"""Symmetric peer-memory heap over NVLink / NVSwitch.

Every rank of a group allocates one device buffer of the same size (CUDA
``cudaMalloc``), exports it as a CUDA IPC handle, and opens every peer's
handle.  Kernels then read and write peers' buffers with plain loads/stores
and signal with system-scope atomics; no library call sits on the data path.
A layout (:class:`HeapLayout`) assigns every region the same offset on all
ranks, so ``peer_ptr(rank, region)`` is the address of ``region`` in
``rank``'s buffer as seen from this process.

Peer pointers are only ever dereferenced by plain ld/st/atom instructions;
no TMA load with cluster multicast ever reads them.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

ALIGN = 256


@dataclass
class Region:
    name: str
    offset: int
    nbytes: int
    shape: tuple[int, ...]
    dtype: torch.dtype


@dataclass
class HeapLayout:
    """Byte layout shared by all ranks (pure Python; CPU-testable)."""

    regions: dict[str, Region] = field(default_factory=dict)
    size: int = 0

    def add(self, name: str, shape: tuple[int, ...], dtype: torch.dtype) -> Region:
        if name in self.regions:
            raise ValueError(f"region {name!r} already defined")
        elem = torch.empty((), dtype=dtype).element_size()
        n = elem
        for d in shape:
            n *= int(d)
        off = (self.size + ALIGN - 1) // ALIGN * ALIGN
        reg = Region(name, off, n, tuple(int(d) for d in shape), dtype)
        self.regions[name] = reg
        self.size = off + n
        return reg

    def __getitem__(self, name: str) -> Region:
        return self.regions[name]


class SymmetricHeap:
    """Collective constructor over ``group`` (every member passes the same layout)."""

    def __init__(self, layout: HeapLayout, *, group=None, device: int | None = None):
        from afd_plugin_b200.ops._ext import ops as cuda_ops

        self.layout = layout
        self.group = group
        self.device = torch.cuda.current_device() if device is None else device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        C = cuda_ops()
        nbytes = max(ALIGN, (layout.size + ALIGN - 1) // ALIGN * ALIGN)
        self.buffer = C.ipc_alloc(nbytes, self.device)
        handle = C.ipc_handle(self.buffer).tolist()
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.base_ptrs: list[int] = []
        self._opened: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.base_ptrs.append(self.buffer.data_ptr())
            else:
                p = C.ipc_open(torch.tensor(h, dtype=torch.uint8), self.device)
                self.base_ptrs.append(p)
                self._opened.append(p)
        dist.barrier(group=group)

    def view(self, name: str) -> torch.Tensor:
        """This rank's copy of region ``name`` as a typed tensor."""
        reg = self.layout[name]
        raw = self.buffer[reg.offset : reg.offset + reg.nbytes]
        return raw.view(reg.dtype).view(reg.shape)

    def peer_ptr(self, rank: int, name: str, extra_offset: int = 0) -> int:
        return self.base_ptrs[rank] + self.layout[name].offset + extra_offset

    def ptr_table(self, ranks: list[int], name: str, extra_offset: int = 0) -> torch.Tensor:
        """int64 device tensor of ``peer_ptr(r, name)`` for ``r`` in ``ranks``."""
        vals = [self.peer_ptr(r, name, extra_offset) for r in ranks]
        return torch.tensor(vals, dtype=torch.int64, device=torch.device("cuda", self.device))

    def close(self) -> None:
        from afd_plugin_b200.ops._ext import ops as cuda_ops

        for p in self._opened:
            try:
                cuda_ops().ipc_close(p, self.device)
            except RuntimeError:
                pass
        self._opened.clear()


__all__ = ["ALIGN", "HeapLayout", "Region", "SymmetricHeap"]
