"""Fail-fast stack validation and the connector factory (CPU, no process group)."""

from __future__ import annotations

from dataclasses import replace

import pytest
import torch

from afd_plugin_b200.config import afd_config_from_mapping
from afd_plugin_b200.connectors.factory import AFDConnectorFactory
from afd_plugin_b200.engine_config import EngineConfig, ModelConfig, ParallelConfig
from afd_plugin_b200.models import get_preset
from afd_plugin_b200.validation import AFD_ATTENTION_WORKER_QUALNAME, AFD_FFN_WORKER_QUALNAME, assert_compatible_afd_stack


def _ec(preset="tiny-dsv2", **par):
    return EngineConfig(ModelConfig(get_preset(preset), dtype=torch.float32, enforce_eager=True),
                        parallel_config=ParallelConfig(**par))


def _afd(**kw):
    return afd_config_from_mapping(dict({"role": "attention", "num_attention_ranks": 2, "num_ffn_ranks": 1}, **kw))


def test_valid_stacks_pass():
    assert_compatible_afd_stack(_ec(data_parallel_size=2), _afd(), worker_cls=AFD_ATTENTION_WORKER_QUALNAME)
    assert_compatible_afd_stack(_ec(data_parallel_size=1, tensor_parallel_size=2), _afd())
    assert_compatible_afd_stack(_ec(), _afd(role="ffn"), worker_cls=AFD_FFN_WORKER_QUALNAME)
    assert_compatible_afd_stack(_ec(data_parallel_size=2, use_ubatching=True, num_ubatches=2), _afd())


@pytest.mark.parametrize("par,afd,message", [
    ({"pipeline_parallel_size": 2}, {}, "pipeline parallelism"),
    ({"use_sequence_parallel_moe": True}, {}, "sequence-parallel MoE"),
    ({"enable_eplb": True}, {}, "EPLB"),
    ({"use_ubatching": True, "num_ubatches": 3}, {}, "exactly two ubatches"),
    ({"data_parallel_size": 3}, {}, "num_attention_ranks=2 must equal"),
    ({}, {"connector": "CAMAsyncAFDConnector", "async": True}, "Ascend-only"),
])
def test_unsupported_stacks_fail_fast(par, afd, message):
    ec = _ec(**{"data_parallel_size": 2, **par})
    with pytest.raises(ValueError, match=message):
        assert_compatible_afd_stack(ec, _afd(**afd))


def test_elastic_ep_and_model_specific_rules():
    ec = _ec(data_parallel_size=2)
    ec.parallel_config.enable_elastic_ep = True  # a field only some stacks carry
    with pytest.raises(ValueError, match="elastic"):
        assert_compatible_afd_stack(ec, _afd())
    with pytest.raises(ValueError, match="compute_gate_on_attention=false"):
        assert_compatible_afd_stack(_ec("tiny-qwen3-moe", data_parallel_size=2), _afd(compute_gate_on_attention=True))
    dense = EngineConfig(ModelConfig(replace(get_preset("tiny-dsv2"), n_routed_experts=0), dtype=torch.float32,
                                     enforce_eager=True), parallel_config=ParallelConfig(data_parallel_size=2))
    with pytest.raises(ValueError, match="requires a MoE model"):
        assert_compatible_afd_stack(dense, _afd(compute_gate_on_attention=True))


def test_worker_class_must_match_the_role():
    with pytest.raises(ValueError, match="requires worker_cls"):
        assert_compatible_afd_stack(_ec(data_parallel_size=2), _afd(), worker_cls=AFD_FFN_WORKER_QUALNAME)


def test_graph_mode_must_be_full_decode_only():
    ec = _ec(data_parallel_size=2)
    ec.model_config.enforce_eager = False
    ec.compilation_config.cudagraph_mode = "PIECEWISE"
    with pytest.raises(RuntimeError, match="FULL_DECODE_ONLY"):
        assert_compatible_afd_stack(ec, _afd())


def test_factory_registry():
    assert {"P2pNcclAFDConnector", "B200FusedAFDConnector"} <= set(AFDConnectorFactory.registered())
    with pytest.raises(ValueError, match="unsupported AFD connector"):
        AFDConnectorFactory.get_connector_class("DummyConnector")
    with pytest.raises(RuntimeError, match="not available on B200"):
        AFDConnectorFactory.get_connector_class("CAMP2pAFDConnector")
    with pytest.raises(ValueError, match="already registered"):
        AFDConnectorFactory.register_connector("P2pNcclAFDConnector", "x", "y")
    p2p = AFDConnectorFactory.get_connector_class("P2pNcclAFDConnector")
    assert p2p.__name__ == "P2pNcclAFDConnector"
    with pytest.raises(ValueError, match="does not support connector_extra_config"):
        p2p.parse_extra_config({"anything": 1})
    fused = AFDConnectorFactory.get_connector_class("B200FusedAFDConnector")
    with pytest.raises(ValueError):
        fused.parse_extra_config({"max_tokens_per_rank": 64, "bogus": 1})
