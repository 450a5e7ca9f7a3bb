"""Process-group plumbing for AFD worlds.

The reference builds a private c10d group next to vLLM's world
(``afd_plugin/distributed/afd_process_group.py:61-116``).  This framework owns
its processes, so the AFD world *is* the default ``torch.distributed`` world
(launched by ``torchrun`` or :mod:`afd_plugin_b200.runtime.launcher`); extra
groups are ordinary ``new_group`` calls.  Timeouts are short by default so a
missing peer surfaces as an error rather than a hang.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT = timedelta(seconds=int(os.environ.get("AFD_B200_PG_TIMEOUT_S", "120")))


def init_afd_world(
    *,
    backend: str | None = None,
    host: str | None = None,
    port: int | None = None,
    world_size: int | None = None,
    rank: int | None = None,
    timeout: timedelta = DEFAULT_TIMEOUT,
    device_id: int | None = None,
) -> tuple[int, int]:
    """Initialise (once) the default group for the AFD world; return ``(rank, size)``.

    With no arguments the ``torchrun`` environment (``RANK``/``WORLD_SIZE``/
    ``MASTER_ADDR``/``MASTER_PORT``) is used.
    """
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kwargs: dict = {"backend": backend, "timeout": timeout}
    if host is not None and port is not None:
        kwargs["init_method"] = f"tcp://{host}:{port}"
        kwargs["world_size"] = int(world_size if world_size is not None else os.environ["WORLD_SIZE"])
        kwargs["rank"] = int(rank if rank is not None else os.environ["RANK"])
    if backend == "nccl" and device_id is not None:
        kwargs["device_id"] = torch.device("cuda", device_id)
    dist.init_process_group(**kwargs)
    return dist.get_rank(), dist.get_world_size()


def new_subgroup(ranks: list[int] | tuple[int, ...], *, backend: str | None = None, timeout: timedelta = DEFAULT_TIMEOUT):
    """Collective: every world rank must call this with the same ``ranks``."""
    return dist.new_group(ranks=list(ranks), backend=backend, timeout=timeout)


def destroy_afd_world() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


__all__ = ["DEFAULT_TIMEOUT", "destroy_afd_world", "init_afd_world", "new_subgroup"]
