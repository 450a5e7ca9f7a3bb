"""Debug-mode validation of the index tensors the kernels trust.

The decode kernels read block tables, sequence lengths, cache slots, state
slots and expert ids without bounds checks: an out-of-range entry would make
them read or write outside their buffers.  With ``AFD_DEBUG_CHECKS=1`` in the
environment (or :func:`enable`), every op entry point in
:mod:`afd_plugin_b200.ops` copies those tensors to the host before the launch
and raises :class:`KernelInputError` naming the first bad entry, so a bad
batch fails on the host instead of faulting the device.  Off by default: the
copies synchronise the stream.  Checks are skipped while a CUDA graph is
being captured (a host copy cannot be captured); replays reuse the buffers
the eager warm-up passes already checked.
"""

from __future__ import annotations

import os

import torch

ENV = "AFD_DEBUG_CHECKS"
_enabled = os.environ.get(ENV, "").strip().lower() in ("1", "true", "yes", "on")


class KernelInputError(ValueError):
    """An index tensor handed to a kernel points outside its buffer."""


def enable(flag: bool = True) -> None:
    global _enabled
    _enabled = bool(flag)


def enabled() -> bool:
    return _enabled


def _active(t: torch.Tensor) -> bool:
    return _enabled and not (t.is_cuda and torch.cuda.is_current_stream_capturing())


def _first_bad(mask: torch.Tensor) -> tuple[int, ...] | None:
    idx = mask.nonzero()
    return tuple(int(i) for i in idx[0]) if idx.numel() else None


def paged_attention(op: str, block_table: torch.Tensor, seq_lens: torch.Tensor, *, num_blocks: int,
                    block_size: int) -> None:
    """Every block a sequence reaches is a real block; lengths fit the table."""
    if not _active(block_table):
        return
    bt = block_table.detach().to("cpu", torch.int64)
    sl = seq_lens.detach().to("cpu", torch.int64).view(-1)
    if bt.dim() != 2 or bt.shape[0] < sl.shape[0]:
        raise KernelInputError(f"{op}: block table {tuple(bt.shape)} has fewer rows than {sl.shape[0]} sequences")
    bad = _first_bad((sl < 1) | (sl > bt.shape[1] * block_size))
    if bad is not None:
        raise KernelInputError(f"{op}: seq_lens[{bad[0]}] = {int(sl[bad[0]])} outside [1, "
                               f"{bt.shape[1] * block_size}] (table width {bt.shape[1]} x block {block_size})")
    used = torch.arange(bt.shape[1])[None, :] < ((sl + block_size - 1) // block_size)[:, None]
    rows = bt[: sl.shape[0]]
    bad = _first_bad(used & ((rows < 0) | (rows >= num_blocks)))
    if bad is not None:
        raise KernelInputError(f"{op}: block_table[{bad[0]}, {bad[1]}] = {int(rows[bad])} outside "
                               f"[0, {num_blocks})")


def cache_slots(op: str, slot_mapping: torch.Tensor, *, num_slots: int) -> None:
    if not _active(slot_mapping):
        return
    s = slot_mapping.detach().to("cpu", torch.int64).view(-1)
    bad = _first_bad((s < 0) | (s >= num_slots))
    if bad is not None:
        raise KernelInputError(f"{op}: slot_mapping[{bad[0]}] = {int(s[bad[0]])} outside [0, {num_slots})")


def state_slots(op: str, slots: torch.Tensor, *, max_seqs: int) -> None:
    if not _active(slots):
        return
    s = slots.detach().to("cpu", torch.int64).view(-1)
    bad = _first_bad((s < 0) | (s >= max_seqs))
    if bad is not None:
        raise KernelInputError(f"{op}: state slot [{bad[0]}] = {int(s[bad[0]])} outside [0, {max_seqs})")


def expert_ids(op: str, ids: torch.Tensor, *, num_experts: int | None = None,
               weights: torch.Tensor | None = None) -> None:
    """Expert ids are non-negative (below ``num_experts`` when given); routing weights are finite."""
    if not _active(ids):
        return
    e = ids.detach().to("cpu", torch.int64)
    hi = num_experts if num_experts is not None else torch.iinfo(torch.int32).max
    bad = _first_bad((e < 0) | (e >= hi))
    if bad is not None:
        raise KernelInputError(f"{op}: expert id at {bad} = {int(e[bad])} outside [0, {hi})")
    if weights is not None:
        w = weights.detach().float().cpu()
        bad = _first_bad(~torch.isfinite(w))
        if bad is not None:
            raise KernelInputError(f"{op}: routing weight at {bad} is {float(w[bad])}")


__all__ = ["ENV", "KernelInputError", "cache_slots", "enable", "enabled", "expert_ids", "paged_attention",
           "state_slots"]
