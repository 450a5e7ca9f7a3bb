"""Wire contract of the reference-semantics connector, with recording fakes (no process group).

The transport calls (``_send`` / ``_recv``) are replaced by recorders, as the
reference's unit tests do (``tests/unit/connectors/test_p2p_connector.py``),
so the order, peers and shapes of every message can be checked on one CPU
process.
"""

import torch

from afd_plugin_b200.config import afd_config_from_mapping
from afd_plugin_b200.connectors.metadata import (
    AFDControlPayload,
    AFDDPMetadata,
    AFDTransferContext,
    AFDTransferMetadata,
)
from afd_plugin_b200.connectors.p2p_nccl import P2pNcclAFDConnector
from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import get_preset

H = get_preset("tiny-dsv2").hidden_size


def _connector(role, role_rank, A=6, F=2):
    afd = afd_config_from_mapping({"role": role, "num_attention_ranks": A, "num_ffn_ranks": F})
    ec = EngineConfig(ModelConfig(get_preset("tiny-dsv2"), dtype=torch.float32), additional_config={"afd": {}})
    c = P2pNcclAFDConnector(0, 0, ec, afd, role_rank)
    c._initialized = True
    log = []

    def send(t, dst):
        log.append(("send", dst, tuple(t.shape), t.dtype))

    def recv(src, spec, ref_tensor=None):
        log.append(("recv", src, tuple(spec.size), spec.dtype))
        return torch.full(tuple(spec.size), float(src), dtype=spec.dtype)

    c._send, c._recv, c.flush = send, recv, lambda: None
    return c, log


def _payload(counts, stages=(0,)):
    return AFDControlPayload(dp_metadata_list={s: AFDDPMetadata(num_tokens_across_dp_cpu=torch.tensor(counts))
                                               for s in stages}, is_graph_capturing=False, is_warmup=False)


def test_attention_rank_sends_hidden_then_ids_to_its_ffn_rank():
    c, log = _connector("attention", 4)  # A4 belongs to FFN rank 1's subgroup (ratio 3)
    counts = [3, 4, 5, 6, 7, 8]
    c.control_plane.update_state_from_dp_metadata(_payload(counts))
    h = torch.zeros(7, H)
    ctx = AFDTransferContext(metadata=AFDTransferMetadata.create_attention_metadata(layer_idx=0, stage_idx=0,
                                                                                   seq_len=7))
    c.send_attn_output(h, ctx, input_ids=torch.arange(7, dtype=torch.int32))
    assert log == [("send", 0, (7, H), torch.float32), ("send", 0, (7,), torch.int32)]
    out = c.recv_ffn_output(ref_tensor=torch.empty(7, H), ubatch_idx=0)
    assert log[-1] == ("recv", 0, (7, H), torch.float32) and out.shape == (7, H)


def test_ffn_rank_fans_in_its_attention_ranks_in_order_and_splits_the_answer():
    c, log = _connector("ffn", 1)  # FFN rank 1 serves A3, A4, A5
    counts = [3, 4, 5, 6, 7, 8]
    c.control_plane.update_state_from_dp_metadata(_payload(counts))
    got = c.recv_attn_output(ubatch_idx=0)
    assert [e[:3] for e in log] == [("recv", 1, (6, H)), ("recv", 2, (7, H)), ("recv", 3, (8, H))]
    assert got.hidden_states.shape == (21, H)
    assert got.context.metadata.seq_lens == [6, 7, 8]
    # rows come back in source order: A3 gets the first 6, A4 the next 7, A5 the last 8
    assert torch.equal(got.hidden_states[:6], torch.ones(6, H)) and torch.equal(got.hidden_states[6:13],
                                                                                  torch.full((7, H), 2.0))
    log.clear()
    c.send_ffn_output(got.hidden_states, got.context)
    assert [e[:3] for e in log] == [("send", 1, (6, H)), ("send", 2, (7, H)), ("send", 3, (8, H))]


def test_ffn_rank_receives_router_logits_and_ids_when_asked():
    from afd_plugin_b200.connectors.metadata import AFDExpertRoutingSpec

    c, log = _connector("ffn", 0, A=2, F=1)
    c.control_plane.update_state_from_dp_metadata(_payload([2, 3]))
    spec = AFDExpertRoutingSpec(router_logits_width=8, router_logits_dtype=torch.float32)
    got = c.recv_attn_output(ubatch_idx=0, routing_spec=spec, recv_input_ids=True)
    # per source: hidden, logits, ids -- then the next source
    assert [(e[1], e[2]) for e in log] == [(1, (2, H)), (1, (2, 8)), (1, (2,)), (2, (3, H)), (2, (3, 8)), (2, (3,))]
    assert got.router_logits.shape == (5, 8) and got.input_ids.shape == (5,)


def test_zero_token_peer_still_sends_one_placeholder_row():
    c, log = _connector("ffn", 0, A=2, F=1)
    c.control_plane.update_state_from_dp_metadata(_payload([0, 4]))
    c.recv_attn_output(ubatch_idx=0)
    assert [e[2] for e in log] == [(1, H), (4, H)]
