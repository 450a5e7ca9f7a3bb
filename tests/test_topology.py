"""Rank placement (behaviour of afd_plugin/distributed/topology.py)."""

from types import SimpleNamespace

import pytest

from afd_plugin_b200.config import afd_config_from_mapping
from afd_plugin_b200.parallel.topology import build_rank_mapping, resolve_role_rank, role_of_world_rank


def cfg(A, F, role="attention"):
    return afd_config_from_mapping({"num_attention_ranks": A, "num_ffn_ranks": F, "role": role})


@pytest.mark.parametrize("A,F", [(1, 1), (2, 2), (3, 1), (4, 2), (6, 2), (4, 4)])
def test_subgroups_partition_world(A, F):
    seen = set()
    for f in range(F):
        m = build_rank_mapping(cfg(A, F, "ffn"), f)
        assert m.world_rank == f and m.subgroup_ranks[0] == f and m.rank_in_subgroup == 0
        assert len(m.subgroup_ranks) == A // F + 1
        seen.update(m.subgroup_ranks[1:])
    assert seen == set(range(F, F + A))
    for a in range(A):
        m = build_rank_mapping(cfg(A, F), a)
        assert m.world_rank == F + a
        assert m.subgroup_index == a // (A // F)
        assert m.subgroup_ranks[m.rank_in_subgroup] == m.world_rank
        assert role_of_world_rank(m.world_rank, attention_size=A, ffn_size=F) == ("attention", a)


def test_6a2f_details():
    m = build_rank_mapping(cfg(6, 2), 4)
    assert m.world_rank == 6 and m.subgroup_index == 1 and m.subgroup_ranks == (1, 5, 6, 7)
    assert m.p2p_rank == 6 and not m.participates_in_dp_metadata_group
    top = build_rank_mapping(cfg(6, 2), 1)
    assert top.participates_in_dp_metadata_group and top.dp_metadata_destinations == (1,)
    f1 = build_rank_mapping(cfg(6, 2, "ffn"), 1)
    assert f1.control_source() == 3


def test_metadata_destinations_fan_out():
    # A >= F always, so each of the first min ranks feeds exactly one FFN rank.
    for a in range(2):
        assert build_rank_mapping(cfg(4, 2), a).dp_metadata_destinations == (a,)


def test_errors():
    with pytest.raises(ValueError):
        build_rank_mapping(cfg(2, 2), 2)
    with pytest.raises(ValueError):
        build_rank_mapping(cfg(2, 2, "ffn"), 5)
    with pytest.raises(ValueError):
        build_rank_mapping(cfg(2, 2), -1)


def test_resolve_role_rank():
    par = SimpleNamespace(data_parallel_size=2, data_parallel_rank=1, tensor_parallel_size=2,
                          prefill_context_parallel_size=1)
    assert resolve_role_rank(par, cfg(4, 2), tp_rank=1) == 3
    with pytest.raises(ValueError):
        resolve_role_rank(par, cfg(2, 2), tp_rank=1)
