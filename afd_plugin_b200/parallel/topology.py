"""AFD rank placement: FFN-first world order and per-FFN subgroups.

World order is ``[F0 .. F(F-1), A0 .. A(A-1)]``.  With ``r = A // F`` each FFN
rank ``k`` owns the subgroup ``{Fk, A(k*r) .. A(k*r + r - 1)}`` in which it is
subgroup rank 0.  The control-plane group holds every FFN rank plus the first
``min(A, F)`` Attention ranks, and Attention rank ``i < min(A, F)`` forwards
control payloads to FFN ranks ``i, i + min, i + 2*min, ...``.

This layout is a wire contract with the reference
(``afd_plugin/distributed/topology.py:16-177``): deployments that mix launch
scripts written for either stack must agree on which process is which rank.
The B200 fused connector uses the same placement; its peer-memory windows are
indexed by world rank.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

from afd_plugin_b200.config import AFDConfig


@dataclass(frozen=True, slots=True)
class AFDRankMapping:
    role: str
    role_rank: int
    world_rank: int
    p2p_rank: int
    attention_size: int
    ffn_size: int
    min_size: int
    ratio: int
    subgroup_index: int
    rank_in_subgroup: int
    subgroup_ranks: tuple[int, ...]
    dp_metadata_destinations: tuple[int, ...] = field(default_factory=tuple)

    @property
    def world_size(self) -> int:
        return self.attention_size + self.ffn_size

    @property
    def is_attention_top_min_size_rank(self) -> bool:
        return self.ffn_size <= self.world_rank < self.ffn_size + self.min_size

    @property
    def participates_in_dp_metadata_group(self) -> bool:
        return self.world_rank < self.ffn_size or self.is_attention_top_min_size_rank

    @property
    def attention_world_ranks(self) -> tuple[int, ...]:
        return tuple(range(self.ffn_size, self.ffn_size + self.attention_size))

    @property
    def ffn_world_ranks(self) -> tuple[int, ...]:
        return tuple(range(self.ffn_size))

    def home_ffn_rank(self, attention_rank: int) -> int:
        """FFN role rank whose subgroup contains Attention role rank ``attention_rank``."""
        return attention_rank // self.ratio

    def control_source(self) -> int:
        """Control-group rank that sends this FFN rank its per-step payload."""
        return self.p2p_rank % self.min_size + self.ffn_size


def topology_from_config(config: AFDConfig) -> tuple[int, int]:
    return config.num_attention_ranks, config.num_ffn_ranks


def validate_p2p_topology(config: AFDConfig) -> None:
    n_attn, n_ffn = topology_from_config(config)
    if n_attn < n_ffn:
        raise ValueError(
            f"{config.connector} currently requires num_attention_ranks >= "
            f"num_ffn_ranks, got {n_attn} < {n_ffn}"
        )
    if n_attn % n_ffn:
        raise ValueError(
            f"{config.connector} currently requires num_attention_ranks to be a "
            f"multiple of num_ffn_ranks, got {n_attn} and {n_ffn}"
        )


def linear_role_rank(dp_rank: int, pcp_rank: int, tp_rank: int, *, pcp_size: int, tp_size: int) -> int:
    """Linearise (dp, pcp, tp) coordinates exactly as the reference does."""
    return (dp_rank * pcp_size + pcp_rank) * tp_size + tp_rank


def resolve_role_rank(parallel_config: Any, config: AFDConfig, *, pcp_rank: int = 0, tp_rank: int = 0) -> int:
    """Role rank of this worker from its data/context/tensor-parallel coordinates.

    ``parallel_config`` needs ``data_parallel_size``, ``data_parallel_rank`` and
    ``tensor_parallel_size`` (``prefill_context_parallel_size`` optional);
    mirrors ``afd_plugin/distributed/topology.py:68-112``.
    """
    dp_size = int(getattr(parallel_config, "data_parallel_size", 1))
    pcp_size = int(getattr(parallel_config, "prefill_context_parallel_size", 1))
    tp_size = int(getattr(parallel_config, "tensor_parallel_size", 1))
    dp_rank = int(getattr(parallel_config, "data_parallel_rank", 0)) if dp_size > 1 else 0
    pcp_rank = pcp_rank if pcp_size > 1 else 0
    tp_rank = tp_rank if tp_size > 1 else 0
    role_rank = linear_role_rank(dp_rank, pcp_rank, tp_rank, pcp_size=pcp_size, tp_size=tp_size)
    if config.role == "attention":
        role_size = config.num_attention_ranks
    elif config.role == "ffn":
        role_size = config.num_ffn_ranks
    else:
        raise ValueError(f"unknown AFD role {config.role!r}")
    if not 0 <= role_rank < role_size:
        raise ValueError(
            "AFD role rank derived from distributed ranks is out of range: "
            f"role={config.role!r}, dp_rank={dp_rank}, pcp_rank={pcp_rank}, "
            f"tp_rank={tp_rank}, role_size={role_size}"
        )
    return role_rank


def build_rank_mapping(config: AFDConfig, role_rank: int) -> AFDRankMapping:
    validate_p2p_topology(config)
    n_attn, n_ffn = topology_from_config(config)
    if role_rank < 0:
        raise ValueError(f"AFD role rank must be non-negative, got {role_rank}")
    ratio = n_attn // n_ffn
    if config.role == "attention":
        if role_rank >= n_attn:
            raise ValueError(
                f"Attention role rank must be within attention size (rank={role_rank}, size={n_attn})"
            )
        world_rank = n_ffn + role_rank
        group = role_rank // ratio
    elif config.role == "ffn":
        if role_rank >= n_ffn:
            raise ValueError(f"FFN role rank must be within FFN size (rank={role_rank}, size={n_ffn})")
        world_rank = role_rank
        group = role_rank
    else:
        raise ValueError(f"unknown AFD role {config.role!r}")

    min_size = min(n_attn, n_ffn)
    members = (group,) + tuple(n_ffn + group * ratio + i for i in range(ratio))
    p2p_rank = role_rank + min_size if config.role == "attention" else role_rank
    dests: tuple[int, ...] = ()
    if n_ffn <= world_rank < n_ffn + min_size:
        dests = tuple(range(world_rank - n_ffn, n_ffn, min_size))
    return AFDRankMapping(
        role=config.role,
        role_rank=role_rank,
        world_rank=world_rank,
        p2p_rank=p2p_rank,
        attention_size=n_attn,
        ffn_size=n_ffn,
        min_size=min_size,
        ratio=ratio,
        subgroup_index=group,
        rank_in_subgroup=members.index(world_rank),
        subgroup_ranks=members,
        dp_metadata_destinations=dests,
    )


def role_of_world_rank(world_rank: int, *, attention_size: int, ffn_size: int) -> tuple[str, int]:
    """Inverse of the world order: ``world_rank -> (role, role_rank)``."""
    if not 0 <= world_rank < attention_size + ffn_size:
        raise ValueError(f"world rank {world_rank} outside world of {attention_size + ffn_size}")
    if world_rank < ffn_size:
        return "ffn", world_rank
    return "attention", world_rank - ffn_size


__all__ = [
    "AFDRankMapping",
    "build_rank_mapping",
    "linear_role_rank",
    "resolve_role_rank",
    "role_of_world_rank",
    "topology_from_config",
    "validate_p2p_topology",
]
