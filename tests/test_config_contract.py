"""``additional_config["afd"]`` contract: the parse / validation behaviour launch commands rely on."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from afd_plugin_b200.config import (
    AFDConfig,
    afd_config_from_mapping,
    connector_extra_config_from_mapping,
    has_afd_config,
    is_afd_active,
    is_afd_async_dp,
    parse_afd_config,
    parse_optional_afd_config,
)


def test_empty_is_inactive_and_required_parse_says_why():
    assert parse_optional_afd_config({}) is None
    with pytest.raises(ValueError, match="additional_config"):
        parse_afd_config({})


def test_namespace_and_config_objects():
    cfg = parse_afd_config({"afd": {"role": "ffn", "connector": "P2pNcclAFDConnector", "num_attention_ranks": 2,
                                    "num_ffn_ranks": 2}}, expected_role="ffn")
    assert cfg.role == cfg.afd_role == "ffn" and cfg.is_ffn_server and not cfg.is_attention_server
    obj = SimpleNamespace(additional_config={"afd": {"role": "attention", "connector": "P2pNcclAFDConnector"}})
    assert parse_afd_config(obj, expected_role="attention").is_attention_server
    with pytest.raises(AttributeError, match="additional_config"):
        parse_optional_afd_config(object())


@pytest.mark.parametrize("raw,want", [("true", True), (1, True), (0, False), ("false", False)])
def test_gate_flag_coercion(raw, want):
    assert afd_config_from_mapping({"compute_gate_on_attention": raw}).compute_gate_on_attention is want


def test_connector_extra_config_goes_to_the_connector():
    raw = {"connector": "B200FusedAFDConnector", "role": "attention",
           "connector_extra_config": {"max_tokens_per_rank": 64}}
    assert connector_extra_config_from_mapping(raw) == {"max_tokens_per_rank": 64}


def test_field_aliases():
    cfg = afd_config_from_mapping({"afd_role": "ffn", "afd_connector": "P2pNcclAFDConnector",
                                   "afd_host": "localhost", "afd_port": 2345})
    assert (cfg.role, cfg.connector, cfg.afd_host, cfg.afd_port) == ("ffn", "P2pNcclAFDConnector", "localhost", 2345)


def test_async_alias_parses_and_needs_the_async_connector():
    cfg = parse_afd_config({"afd": {"connector": "CAMAsyncAFDConnector", "role": "attention", "async": "true"}})
    assert cfg.async_dp is True
    with pytest.raises(ValueError, match="CAMAsyncAFDConnector"):
        parse_afd_config({"afd": {"connector": "CAMP2pAFDConnector", "role": "attention", "async": True}})


def test_presence_versus_activation():
    bad_role = {"afd": {"role": "decode"}}
    assert has_afd_config(bad_role) is True
    with pytest.raises(ValueError, match="AFD role must be one of"):
        is_afd_active(bad_role)
    assert is_afd_active({"afd": {"role": "attention"}}) is True
    assert is_afd_active({}) is False
    selector = {"afd": {"connector": "CAMAsyncAFDConnector", "async": True, "role": "decode"}}
    assert is_afd_async_dp(SimpleNamespace(additional_config=selector)) is True


def test_integer_fields():
    class IntLike:
        def __int__(self) -> int:
            return 2

    cfg = afd_config_from_mapping({"num_attention_ranks": IntLike(), "num_ffn_ranks": IntLike()})
    assert (cfg.num_attention_ranks, cfg.num_ffn_ranks) == (2, 2)
    with pytest.raises(TypeError, match="num_attention_ranks must be an integer"):
        afd_config_from_mapping({"num_attention_ranks": 2.5})


@pytest.mark.parametrize("raw,message", [
    ({"enabled": True}, "unknown AFD config field"),
    ({"role": "decode"}, "AFD role must be one of"),
    ({"connector": "tcp"}, "AFD connector must be one of"),
    ({"afd_role_rank": 0}, "unknown AFD config field"),
    ({"num_attention_servers": 2}, "unknown AFD config field"),
    ({"afd_server_rank": 0}, "unknown AFD config field"),
])
def test_clear_errors(raw, message):
    with pytest.raises((TypeError, ValueError), match=message):
        afd_config_from_mapping(raw)


def test_role_mismatch_and_hash():
    with pytest.raises(ValueError, match="AFD role mismatch"):
        afd_config_from_mapping({"role": "ffn"}, expected_role="attention")
    assert AFDConfig(role="attention").compute_hash() != AFDConfig(role="ffn").compute_hash()
