"""FFN-role model runner and its connector-driven serving loop.

Per control payload the runner walks ``layers x stages``:
``recv_attn_output -> compute -> send_ffn_output`` -- the structure of
``GPUFFNModelRunner._ffn_forward`` (``afd_plugin/v1/worker/ffn_model_runner.py:167-247``).
Graphs are cached by :func:`count_graph_key` and replayed when the
Attention side replays (:func:`pick_run_mode`).

With several FFN ranks the routed experts are sharded (expert parallelism):
for MoE layers each FFN rank gathers its peers' tokens, applies its local
experts to all of them and the partial outputs are reduced back to the owning
rank -- the all-gather / reduce-scatter exchange vLLM's FusedMoE performs in
the reference deployment.  Shared experts run on the owning rank only.
"""

from __future__ import annotations

import logging
import threading
from typing import Any

import torch
import torch.distributed as dist

from afd_plugin_b200.connectors.metadata import AFDControlPayload
from afd_plugin_b200.runtime.cuda_graph import (
    RunMode,
    count_graph_key,
    graph_settings,
    pick_run_mode,
)
from afd_plugin_b200.runtime.ffn_metadata import aggregate_ffn_token_counts

log = logging.getLogger(__name__)


class FFNModelRunner:
    def __init__(self, model, connector, engine_config, *, ep_group=None, ep_size: int = 1, ep_rank: int = 0):
        self.model = model
        self.connector = connector
        self.config = engine_config
        self.ep_group = ep_group
        self.ep_size = ep_size
        self.ep_rank = ep_rank
        self.device = model.device
        policy = graph_settings(engine_config, role="ffn")
        self.use_cuda_graph = policy.enabled and self.device.type == "cuda" and self._graph_capable()
        self._graphs: dict[tuple, dict[str, Any]] = {}
        self._pool = None
        self._ffn_counts: dict[int, tuple[int, ...]] = {}
        self.steps = 0
        # Set by benchmarks: count the kernels of the next eager step.
        self.count_next_eager = False
        self.kernels_per_step = 0

    def _graph_capable(self) -> bool:
        return bool(getattr(self.connector, "supports_graph_capture", False))

    # ----------------------------------------------------------- stepping
    def execute_model(self, payload: AFDControlPayload) -> None:
        dpl = payload.dp_metadata_list
        key = count_graph_key(dpl, attention_size=self.connector.attn_size, ffn_size=self.connector.ffn_size)
        entry = self._graphs.get(key)
        mode = pick_run_mode(
            warmup=payload.is_warmup,
            capturing=payload.is_graph_capturing,
            replaying=payload.is_graph_replaying,
            graphs_on=self.use_cuda_graph,
            have_graph=entry is not None,
        )
        self.steps += 1
        if mode is RunMode.REPLAY:
            self.connector.control_plane.update_state_from_dp_metadata(payload)
            entry["graph"].replay()
            return
        if mode is RunMode.CAPTURE and self.use_cuda_graph:
            self._capture(payload, key)
            return
        if self.count_next_eager and mode is RunMode.EAGER and self.device.type == "cuda":
            from afd_plugin_b200.utils.launch_count import count_afd_kernels

            self.count_next_eager = False
            self.kernels_per_step = count_afd_kernels(lambda: self._ffn_forward(payload))
            return
        self._ffn_forward(payload)

    def _capture(self, payload: AFDControlPayload, key) -> None:
        self.connector.control_plane.update_state_from_dp_metadata(payload)
        graph = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        with torch.profiler.record_function(f"ffn_capture_{key}"), torch.cuda.graph(graph, pool=self._pool):
            self._ffn_forward(payload, update_state=False)
        self._graphs[key] = {"graph": graph}

    def _ffn_forward(self, payload: AFDControlPayload, *, update_state: bool = True) -> torch.Tensor | None:
        c = self.connector
        if update_state:
            c.control_plane.update_state_from_dp_metadata(payload)
        stages = sorted(payload.dp_metadata_list) or [0]
        self._ffn_counts = {
            s: aggregate_ffn_token_counts(
                tuple(int(x) for x in payload.dp_metadata_list[s].num_tokens_across_dp_cpu.tolist()),
                attention_size=c.attn_size, ffn_size=c.ffn_size)
            for s in stages
        }
        model = self.model
        gate_on_attn = model.compute_gate_on_attention
        out = None
        for layer in model.ffn_layer_indices():
            is_moe = model.arch.is_moe_layer(layer)
            routing_spec = model.get_experts_routing_spec(layer) if (is_moe and gate_on_attn) else None
            want_ids = model.ffn_needs_input_ids(layer)
            for stage in stages:
                kw = {"routing_spec": routing_spec} if routing_spec is not None else {}
                if want_ids:
                    kw["recv_input_ids"] = True
                recv = c.recv_attn_output(ubatch_idx=stage, **kw)
                recv.context.metadata.layer_idx = layer
                recv.context.metadata.stage_idx = stage
                out = self.compute(layer, stage, recv.hidden_states, recv.router_logits, recv.input_ids)
                c.send_ffn_output(out, recv.context)
        flush = getattr(c, "flush", None)
        if callable(flush):
            flush()
        return out

    # ------------------------------------------------------------ compute
    def compute(self, layer: int, stage: int, h: torch.Tensor, router_logits: torch.Tensor | None,
                input_ids: torch.Tensor | None = None) -> torch.Tensor:
        model = self.model
        if not model.arch.is_moe_layer(layer):
            return model.compute_ffn_output(h, layer)
        if self.ep_size == 1:
            if router_logits is not None:
                return model.compute_experts_output(h, layer, router_logits)
            return model.compute_ffn_output(h, layer, input_ids=input_ids)
        return self._moe_expert_parallel(layer, stage, h, router_logits, input_ids)

    def _moe_expert_parallel(self, layer: int, stage: int, h: torch.Tensor, router_logits,
                             input_ids: torch.Tensor | None = None) -> torch.Tensor:
        moe = self.model.layers[layer].mlp
        counts = self._ffn_counts[stage]
        n_max = max(counts)
        H = h.shape[1]

        def gather(x: torch.Tensor) -> torch.Tensor:
            pad = x.new_zeros((n_max, x.shape[1]))
            pad[: x.shape[0]] = x
            parts = [torch.empty_like(pad) for _ in range(self.ep_size)]
            dist.all_gather(parts, pad, group=self.ep_group)
            return torch.cat([p[:n] for p, n in zip(parts, counts)], dim=0)

        h_all = gather(h)
        logits_all = gather(router_logits) if router_logits is not None else moe.gate.logits(h_all)
        ids_all = gather(input_ids.view(-1, 1)).view(-1) if input_ids is not None else None
        w, ids = moe.gate.route(logits_all, ids_all)
        partial = moe.experts(h_all, w, ids).float()
        # Reduce the partial sums back to their owners.
        padded = partial.new_zeros((self.ep_size * n_max, H))
        off = 0
        for r, n in enumerate(counts):
            padded[r * n_max : r * n_max + n] = partial[off : off + n]
            off += n
        if dist.get_backend(self.ep_group) == "nccl":
            mine = padded.new_empty((n_max, H))
            dist.reduce_scatter_tensor(mine, padded, group=self.ep_group)
        else:
            dist.all_reduce(padded, group=self.ep_group)
            mine = padded[self.ep_rank * n_max : (self.ep_rank + 1) * n_max]
        out = mine[: h.shape[0]].to(h.dtype)
        if moe.shared_experts is not None:
            shared = moe.shared_experts(h)
            sg = moe.shared_gate(h)
            out = out + (shared if sg is None else (shared.float() * sg).to(shared.dtype))
        return out

    # ------------------------------------------------------------ serving
    def serve(self, *, max_steps: int | None = None, stop: threading.Event | None = None) -> int:
        """Run steps until a shutdown payload, ``max_steps`` or ``stop``; returns steps run."""
        cp = self.connector.control_plane
        if cp is None:
            raise NotImplementedError("FFN serving needs a control-plane-driven connector")
        from afd_plugin_b200.utils.profiler import RoleProfiler

        prof = RoleProfiler("ffn")
        n = 0
        try:
            while (max_steps is None or n < max_steps) and not (stop is not None and stop.is_set()):
                check = getattr(self, "health_check", None)
                if check is not None:
                    check()  # a peer stopped heartbeating: fail before waiting on it
                payload = cp.recv_dp_metadata_list()
                if payload.is_shutdown:
                    break
                self.execute_model(payload)
                if self.device.type == "cuda":
                    torch.cuda.synchronize(self.device)
                n += 1
                prof.step()
        finally:
            prof.close()
        return n

    def release_graphs(self) -> None:
        self._graphs.clear()
        self._pool = None

    def reload_weights(self, checkpoint: str | None = None, *, seed: int = 0) -> None:
        """Reload the FFN weights in place between steps (``ffn_model_runner.py:288-291``).

        Parameters keep their storage, so cached graphs replay the new weights.
        """
        self.model.reload_weights(checkpoint, seed=seed)


__all__ = ["FFNModelRunner"]
