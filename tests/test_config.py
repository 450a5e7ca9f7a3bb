"""AFD config parsing/validation (behaviour of afd_plugin/config.py)."""

from types import SimpleNamespace

import pytest

from afd_plugin_b200.config import (
    AFDConfig,
    afd_config_from_mapping,
    connector_extra_config_from_source,
    has_afd_config,
    is_afd_active,
    is_afd_async_dp,
    parse_afd_config,
    parse_optional_afd_config,
)
from afd_plugin_b200.config_utils import (
    coerce_extra_bool,
    coerce_extra_int,
    coerce_extra_positive_int,
    coerce_extra_str,
    coerce_optional_extra_positive_int,
)


def test_defaults():
    c = AFDConfig()
    assert c.connector == "P2pNcclAFDConnector" and c.port == 1239 and c.host == "127.0.0.1"
    assert c.is_attention_server and not c.is_ffn_server
    assert c.afd_role == "attention" and c.afd_port == 1239


def test_aliases_and_coercion():
    c = afd_config_from_mapping({"afd_role": "ffn", "afd_port": "2000", "async": "no", "num_ffn_ranks": 1,
                                 "compute_gate_on_attention": "yes"})
    assert c.role == "ffn" and c.port == 2000 and c.async_dp is False and c.compute_gate_on_attention


def test_unknown_and_duplicate_keys():
    with pytest.raises(ValueError, match="unknown AFD config field"):
        afd_config_from_mapping({"bogus": 1})
    with pytest.raises(ValueError, match="duplicate"):
        afd_config_from_mapping({"role": "ffn", "afd_role": "ffn"})


@pytest.mark.parametrize("bad", [{"role": "x"}, {"port": 0}, {"port": 70000}, {"host": ""},
                                 {"num_attention_ranks": 0}, {"connector": "Nope"},
                                 {"num_attention_ranks": 3, "num_ffn_ranks": 2},
                                 {"num_attention_ranks": 1, "num_ffn_ranks": 2},
                                 {"async": True}])
def test_invalid(bad):
    with pytest.raises(ValueError):
        afd_config_from_mapping(bad)


def test_expected_role():
    with pytest.raises(ValueError, match="role mismatch"):
        afd_config_from_mapping({"role": "ffn"}, expected_role="attention")


def test_sources():
    src = SimpleNamespace(additional_config={"afd": {"role": "ffn", "connector_extra_config": {"k": 1}}})
    assert has_afd_config(src) and is_afd_active(src)
    assert parse_afd_config(src).role == "ffn"
    assert connector_extra_config_from_source(src) == {"k": 1}
    assert parse_optional_afd_config({"other": 1}) is None
    assert not is_afd_async_dp(src)
    with pytest.raises(ValueError):
        parse_afd_config(SimpleNamespace(additional_config={}))
    with pytest.raises(TypeError):
        parse_afd_config(SimpleNamespace(additional_config={"afd": 3}))


def test_hash_stable_and_sensitive():
    a = afd_config_from_mapping({"num_attention_ranks": 2})
    b = afd_config_from_mapping({"num_attention_ranks": 2, "port": 5})
    c = afd_config_from_mapping({"num_attention_ranks": 4})
    assert a.compute_hash() == b.compute_hash() != c.compute_hash()


def test_b200_connector_accepted():
    c = afd_config_from_mapping({"connector": "B200FusedAFDConnector", "num_attention_ranks": 6, "num_ffn_ranks": 2})
    assert c.connector == "B200FusedAFDConnector"


def test_coercions():
    assert coerce_extra_bool(1, field_name="x") is True
    assert coerce_extra_bool("Off", field_name="x") is False
    with pytest.raises(TypeError):
        coerce_extra_bool(2, field_name="x")
    with pytest.raises(TypeError):
        coerce_extra_int(1.5, field_name="x")
    with pytest.raises(TypeError):
        coerce_extra_int(True, field_name="x")
    assert coerce_extra_int("7", field_name="x") == 7
    with pytest.raises(ValueError):
        coerce_extra_positive_int(0, field_name="x")
    assert coerce_optional_extra_positive_int("", field_name="x") is None
    assert coerce_extra_str(" ABC ", field_name="x") == "abc"
