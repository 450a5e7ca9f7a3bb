"""FFN model runner against recording fakes (no process group, no GPU).

Covers the runner contract of ``afd_plugin/v1/worker/ffn_model_runner.py:167-247``:
the ``layers x stages`` walk (recv -> compute -> send per pair, flush once),
per-FFN-rank token aggregation, routing-spec / input-id requests, the CUDA
graph run modes (replay of a cached key, eager fallback when no graph exists,
warm-up and capture falling back to eager when graphs are off) and the FFN
worker's refusal of scheduler-driven ``execute_model``.
"""

from __future__ import annotations

import threading
from types import SimpleNamespace

import pytest
import torch

from afd_plugin_b200.connectors.metadata import AFDControlPayload, AFDDPMetadata, AFDExpertRoutingSpec
from afd_plugin_b200.runtime.cuda_graph import count_graph_key
from afd_plugin_b200.runtime.ffn_runner import FFNModelRunner

H = 8


class FakeArch:
    def __init__(self, moe_layers):
        self.moe_layers = set(moe_layers)

    def is_moe_layer(self, layer):
        return layer in self.moe_layers


class FakeModel:
    def __init__(self, layers=(0, 1, 2), moe_layers=(1, 2), gate_on_attn=False, ids_layers=()):
        self.device = torch.device("cpu")
        self.arch = FakeArch(moe_layers)
        self._layers = tuple(layers)
        self.compute_gate_on_attention = gate_on_attn
        self._ids_layers = set(ids_layers)
        self.calls = []

    def ffn_layer_indices(self):
        return self._layers

    def get_experts_routing_spec(self, layer):
        return AFDExpertRoutingSpec(4, torch.float32)

    def ffn_needs_input_ids(self, layer):
        return layer in self._ids_layers

    def compute_ffn_output(self, h, layer, input_ids=None):
        self.calls.append(("ffn", layer, h.shape[0], None if input_ids is None else input_ids.tolist()))
        return h * (layer + 2)

    def compute_experts_output(self, h, layer, logits):
        self.calls.append(("experts", layer, h.shape[0], tuple(logits.shape)))
        return h + layer


class FakeControlPlane:
    def __init__(self, payloads=()):
        self.updates = []
        self._payloads = list(payloads)

    def update_state_from_dp_metadata(self, payload):
        self.updates.append(payload)

    def recv_dp_metadata_list(self):
        return self._payloads.pop(0)


class FakeConnector:
    def __init__(self, attn_size=2, ffn_size=1, tokens=3, control_plane=None):
        self.attn_size = attn_size
        self.ffn_size = ffn_size
        self.tokens = tokens
        self.control_plane = control_plane or FakeControlPlane()
        self.events = []
        self.flushes = 0

    def recv_attn_output(self, ubatch_idx=0, routing_spec=None, recv_input_ids=False):
        self.events.append(("recv", ubatch_idx, routing_spec is not None, recv_input_ids))
        n = self.tokens + ubatch_idx
        h = torch.full((n, H), float(ubatch_idx + 1))
        logits = torch.zeros(n, routing_spec.router_logits_width) if routing_spec is not None else None
        ids = torch.arange(n) if recv_input_ids else None
        ctx = SimpleNamespace(metadata=SimpleNamespace(layer_idx=-1, stage_idx=-1))
        return SimpleNamespace(hidden_states=h, router_logits=logits, input_ids=ids, context=ctx)

    def send_ffn_output(self, out, ctx):
        self.events.append(("send", ctx.metadata.layer_idx, ctx.metadata.stage_idx, float(out[0, 0])))

    def flush(self):
        self.flushes += 1


def _cfg(eager=True):
    return SimpleNamespace(model_config=SimpleNamespace(enforce_eager=eager),
                           compilation_config=SimpleNamespace(cudagraph_mode="FULL_DECODE_ONLY"),
                           parallel_config=SimpleNamespace(use_ubatching=False))


def _payload(stages=(0,), counts=(3, 3), **flags):
    dpl = {s: AFDDPMetadata(num_tokens_across_dp_cpu=torch.tensor(counts)) for s in stages}
    return AFDControlPayload(dp_metadata_list=dpl, is_graph_capturing=flags.get("capturing", False),
                             is_warmup=flags.get("warmup", False),
                             is_graph_replaying=flags.get("replaying", False),
                             is_shutdown=flags.get("shutdown", False))


def test_layer_stage_walk_order_and_flush():
    model, conn = FakeModel(), FakeConnector()
    runner = FFNModelRunner(model, conn, _cfg())
    runner.execute_model(_payload(stages=(1, 0)))
    recv = [e for e in conn.events if e[0] == "recv"]
    send = [e for e in conn.events if e[0] == "send"]
    # layer-major, stages ascending, each recv followed by its send
    assert [e[1] for e in recv] == [0, 1] * 3
    assert [(e[1], e[2]) for e in send] == [(layer, s) for layer in (0, 1, 2) for s in (0, 1)]
    assert [e[0] for e in conn.events] == ["recv", "send"] * 6
    assert conn.flushes == 1
    assert len(conn.control_plane.updates) == 1
    # dense layer -> compute_ffn_output; MoE layers without logits also use the full FFN path
    assert [c[:2] for c in model.calls] == [("ffn", 0)] * 2 + [("ffn", 1)] * 2 + [("ffn", 2)] * 2
    # output of layer 0 stage 1: hidden 2.0 scaled by (0 + 2)
    assert send[1][3] == 4.0


def test_gate_on_attention_requests_logits_for_moe_layers_only():
    model, conn = FakeModel(gate_on_attn=True), FakeConnector()
    FFNModelRunner(model, conn, _cfg()).execute_model(_payload())
    assert [e[2] for e in conn.events if e[0] == "recv"] == [False, True, True]
    assert [c[0] for c in model.calls] == ["ffn", "experts", "experts"]
    assert model.calls[1][3] == (3, 4)


def test_input_ids_requested_for_hash_layers():
    model, conn = FakeModel(ids_layers=(1,)), FakeConnector()
    FFNModelRunner(model, conn, _cfg()).execute_model(_payload())
    assert [e[3] for e in conn.events if e[0] == "recv"] == [False, True, False]
    assert model.calls[1][3] == [0, 1, 2]


def test_token_counts_aggregated_per_ffn_rank():
    conn = FakeConnector(attn_size=4, ffn_size=2)
    runner = FFNModelRunner(FakeModel(), conn, _cfg())
    runner.execute_model(_payload(stages=(0, 1), counts=(1, 2, 0, 4)))
    # FFN rank k sums Attention ranks k*r..k*r+r-1; an idle rank still sends one placeholder row
    assert runner._ffn_counts == {0: (3, 5), 1: (3, 5)}


class FakeGraph:
    def __init__(self):
        self.replays = 0

    def replay(self):
        self.replays += 1


def test_replay_uses_cached_graph_without_touching_the_connector():
    model, conn = FakeModel(), FakeConnector()
    runner = FFNModelRunner(model, conn, _cfg())
    runner.use_cuda_graph = True
    p = _payload(replaying=True)
    key = count_graph_key(p.dp_metadata_list, attention_size=conn.attn_size, ffn_size=conn.ffn_size)
    g = FakeGraph()
    runner._graphs[key] = {"graph": g}
    runner.execute_model(p)
    assert g.replays == 1
    assert conn.events == [] and model.calls == []
    assert conn.control_plane.updates == [p]


def test_replay_without_graph_or_with_other_key_runs_eagerly():
    model, conn = FakeModel(), FakeConnector()
    runner = FFNModelRunner(model, conn, _cfg())
    runner.use_cuda_graph = True
    g = FakeGraph()
    other = _payload(counts=(5, 5))
    runner._graphs[count_graph_key(other.dp_metadata_list, attention_size=2, ffn_size=1)] = {"graph": g}
    runner.execute_model(_payload(replaying=True))
    assert g.replays == 0
    assert len([e for e in conn.events if e[0] == "recv"]) == 3


@pytest.mark.parametrize("flags", [{"warmup": True}, {"capturing": True}, {}])
def test_warmup_and_capture_run_eagerly_when_graphs_are_off(flags):
    model, conn = FakeModel(), FakeConnector()
    runner = FFNModelRunner(model, conn, _cfg(eager=True))
    assert runner.use_cuda_graph is False
    runner.execute_model(_payload(**flags))
    assert len(model.calls) == 3 and runner._graphs == {}
    assert runner.steps == 1


def test_graphs_need_a_capture_capable_connector_and_cuda():
    conn = FakeConnector()
    runner = FFNModelRunner(FakeModel(), conn, _cfg(eager=False))
    assert runner.use_cuda_graph is False  # CPU device, connector without supports_graph_capture


def test_unsupported_graph_mode_rejected():
    cfg = _cfg(eager=False)
    cfg.compilation_config.cudagraph_mode = "PIECEWISE"
    with pytest.raises(RuntimeError, match="FULL_DECODE_ONLY"):
        FFNModelRunner(FakeModel(), FakeConnector(), cfg)


def test_serve_until_shutdown_payload():
    cp = FakeControlPlane([_payload(), _payload(stages=(0, 1)), _payload(shutdown=True), _payload()])
    conn = FakeConnector(control_plane=cp)
    runner = FFNModelRunner(FakeModel(), conn, _cfg())
    assert runner.serve() == 2
    assert conn.flushes == 2
    assert len(cp._payloads) == 1  # the payload after shutdown is never read


def test_serve_stops_on_event_and_max_steps():
    cp = FakeControlPlane([_payload() for _ in range(5)])
    runner = FFNModelRunner(FakeModel(), FakeConnector(control_plane=cp), _cfg())
    assert runner.serve(max_steps=3) == 3
    stop = threading.Event()
    stop.set()
    assert runner.serve(stop=stop) == 0
    assert len(cp._payloads) == 2


def test_serve_needs_a_control_plane():
    conn = FakeConnector()
    conn.control_plane = None
    runner = FFNModelRunner(FakeModel(), conn, _cfg())
    with pytest.raises(NotImplementedError):
        runner.serve(max_steps=1)


def test_ffn_worker_rejects_scheduler_driven_execute_model():
    from afd_plugin_b200.runtime.workers import AFDFFNWorker

    worker = object.__new__(AFDFFNWorker)
    with pytest.raises(RuntimeError, match="connector-driven"):
        worker.execute_model(None)


def test_reload_weights_delegates_and_worker_refuses_while_serving():
    from afd_plugin_b200.runtime.workers import AFDFFNWorker

    model = FakeModel()
    seen = []
    model.reload_weights = lambda ckpt, seed=0: seen.append((ckpt, seed))
    runner = FFNModelRunner(model, FakeConnector(), _cfg())
    runner.reload_weights("/ckpt", seed=3)
    assert seen == [("/ckpt", 3)]

    worker = object.__new__(AFDFFNWorker)
    worker.config = SimpleNamespace(model_config=SimpleNamespace(checkpoint=None, seed=11))
    worker.model_runner = runner
    release = threading.Event()
    worker._thread = threading.Thread(target=release.wait, daemon=True)
    worker._thread.start()
    try:
        with pytest.raises(RuntimeError, match="stop the FFN server loop"):
            worker.reload_weights()
    finally:
        release.set()
        worker._thread.join()
    worker.reload_weights()
    assert seen[-1] == (None, 11)


def test_attention_side_graphs_follow_the_connector():
    from afd_plugin_b200.runtime.ffn_executor import ConnectorFFNExecutor, LocalFFNExecutor

    model = SimpleNamespace(compute_gate_on_attention=False)
    assert ConnectorFFNExecutor(model, SimpleNamespace()).supports_graph_capture is False
    assert ConnectorFFNExecutor(model, SimpleNamespace(supports_graph_capture=True)).supports_graph_capture
    assert LocalFFNExecutor(model).supports_graph_capture
