"""Control payload codec, transfer metadata, graph policy, FFN token counts."""

from types import SimpleNamespace

import pytest
import torch

from afd_plugin_b200.connectors.metadata import (
    AFDControlPayload,
    AFDDPMetadata,
    AFDTransferMetadata,
    decode_control_payload,
    encode_control_payload,
)
from afd_plugin_b200.runtime.cuda_graph import (
    RunMode,
    capacity_graph_key,
    count_graph_key,
    graph_settings,
    pad_to_capture_size,
    pick_run_mode,
)
from afd_plugin_b200.runtime.ffn_metadata import aggregate_ffn_token_counts, project_ffn_token_counts_to_dp


def test_codec_roundtrip():
    p = AFDControlPayload({0: AFDDPMetadata([3, 4]), 1: AFDDPMetadata([5, 0])}, is_graph_capturing=True,
                          is_warmup=False, is_graph_replaying=True, is_profile=True)
    q = decode_control_payload(encode_control_payload(p))
    assert q.is_graph_capturing and q.is_graph_replaying and q.is_profile and not q.is_warmup
    assert q.dp_metadata_list[1].num_tokens_across_dp_cpu.tolist() == [5, 0]
    assert int(q.dp_metadata_list[0].max_tokens_across_dp_cpu) == 4
    # the wire format is compact sorted JSON
    blob = encode_control_payload(p)
    assert blob.startswith(b'{"dp_metadata_list":')


def test_shutdown_flag_roundtrip():
    p = AFDControlPayload({0: AFDDPMetadata([1])}, False, False, is_shutdown=True)
    assert decode_control_payload(encode_control_payload(p)).is_shutdown


def test_dp_metadata_peak():
    m = AFDDPMetadata([5, 3])
    assert m.num_tokens_across_dp_cpu.dtype == torch.int32 and int(m.max_tokens_across_dp_cpu) == 5
    assert int(AFDDPMetadata([]).max_tokens_across_dp_cpu) == 0


def test_transfer_metadata():
    m = AFDTransferMetadata.create_ffn_metadata(layer_idx=1, stage_idx=0, seq_lens=[2, 3])
    assert m.total_tokens == 5 and m.validate_tensor_shape((5, 8)) and not m.validate_tensor_shape((4, 8))
    with pytest.raises(ValueError):
        AFDTransferMetadata(0, 0, [])
    with pytest.raises(ValueError):
        AFDTransferMetadata(0, 0, [0])


def test_ffn_counts():
    assert aggregate_ffn_token_counts((0, 4, 5, 6), attention_size=4, ffn_size=2) == (5, 11)
    assert aggregate_ffn_token_counts((), attention_size=4, ffn_size=2) == (2, 2)
    assert aggregate_ffn_token_counts((3,), attention_size=2, ffn_size=1) == (6,)
    assert aggregate_ffn_token_counts((1, 2), attention_size=3, ffn_size=2) == (1, 1)
    assert project_ffn_token_counts_to_dp((8, 8, 13, 13), dp_size=2) == (8, 13)
    assert project_ffn_token_counts_to_dp((8, 13), dp_size=2) == (8, 13)


def test_graph_key_and_modes():
    dpl = {1: AFDDPMetadata([1, 2, 3, 4]), 0: AFDDPMetadata([0, 0, 5, 5])}
    assert count_graph_key(dpl) == ((0, (0, 0, 5, 5)), (1, (1, 2, 3, 4)))
    # each FFN rank receives its two peers' rows; an empty peer sends one placeholder row
    assert count_graph_key(dpl, attention_size=4, ffn_size=2) == ((0, (2, 10)), (1, (3, 7)))
    # counts given per DP rank are expanded over TP peers (DP 2 x TP 2 = 4 Attention ranks)
    assert count_graph_key({0: AFDDPMetadata([3, 4])}, attention_size=4, ffn_size=2) == ((0, (6, 8)),)
    assert capacity_graph_key((1, 0), 64) == ("capacity", (0, 1), 64)
    kw = dict(warmup=False, capturing=False, replaying=True, graphs_on=True)
    assert pick_run_mode(have_graph=True, **kw) is RunMode.REPLAY
    assert pick_run_mode(have_graph=False, **kw) is RunMode.EAGER
    assert pick_run_mode(warmup=False, capturing=False, replaying=True, graphs_on=False,
                         have_graph=True) is RunMode.EAGER
    assert pick_run_mode(warmup=True, capturing=True, replaying=True, graphs_on=True,
                         have_graph=True) is RunMode.WARMUP
    assert pick_run_mode(warmup=False, capturing=True, replaying=False, graphs_on=True,
                         have_graph=False) is RunMode.CAPTURE
    assert pad_to_capture_size(5, [8, 4, 16]) == 8 and pad_to_capture_size(17, [8, 16]) is None


def _cfg(eager=False, mode="FULL_DECODE_ONLY", ub=False, n=1):
    return SimpleNamespace(model_config=SimpleNamespace(enforce_eager=eager),
                           compilation_config=SimpleNamespace(cudagraph_mode=mode),
                           parallel_config=SimpleNamespace(use_ubatching=ub, num_ubatches=n))


def test_graph_policy():
    assert not graph_settings(_cfg(eager=True)).enabled
    p = graph_settings(_cfg(ub=True, n=2), role="ffn")
    assert p.enabled and p.ffn_graphs and not p.attention_graphs and p.two_ubatches
    with pytest.raises(RuntimeError, match="FULL_DECODE_ONLY"):
        graph_settings(_cfg(mode="PIECEWISE"))
    with pytest.raises(RuntimeError, match="two ubatches"):
        graph_settings(_cfg(ub=True, n=3))
    enum_like = SimpleNamespace(name="FULL_DECODE_ONLY")
    assert graph_settings(_cfg(mode=enum_like)).mode == "FULL_DECODE_ONLY"
    assert graph_settings(_cfg(mode="CUDAGraphMode.FULL_DECODE_ONLY")).enabled
