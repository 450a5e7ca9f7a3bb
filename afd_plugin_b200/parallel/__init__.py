"""Rank topology, process groups and peer-memory plumbing."""

from afd_plugin_b200.parallel.topology import (
    AFDRankMapping,
    build_rank_mapping,
    linear_role_rank,
    resolve_role_rank,
    role_of_world_rank,
    topology_from_config,
    validate_p2p_topology,
)

__all__ = [
    "AFDRankMapping",
    "build_rank_mapping",
    "linear_role_rank",
    "resolve_role_rank",
    "role_of_world_rank",
    "topology_from_config",
    "validate_p2p_topology",
]
