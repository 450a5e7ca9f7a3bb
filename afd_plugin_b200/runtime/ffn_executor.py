"""Attention-side handling of the FFN boundary of each decoder layer.

The model runner calls ``send(layer, attn_out, residual, stage)`` after a
layer's attention and ``recv(layer, handle, stage)`` before the next layer;
splitting the two lets the DBO scheduler place the other ubatch's attention
between them.

* :class:`LocalFFNExecutor` -- colocated: post-attention norm + local FFN.
* :class:`ConnectorFFNExecutor` -- AFD through a connector with reference
  semantics (``RemoteFFNProxy`` / ``AFDAttentionFusedMoE`` of
  ``afd_plugin/model_executor/models/deepseek_v2.py:112-184``).
* The fused B200 executor lives with its connector
  (:mod:`afd_plugin_b200.connectors.b200_fused`).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from afd_plugin_b200.utils.phase_timer import NULL_TIMER
from afd_plugin_b200.connectors.metadata import (
    AFDControlPayload,
    AFDDPMetadata,
    AFDTransferContext,
    AFDTransferMetadata,
)


class FFNExecutor:
    """Interface; ``begin_step`` is called once per forward before layer 0.

    ``supports_graph_capture``: whether a decode step through this executor
    may be captured into a CUDA graph (the engine runs eagerly otherwise).
    """

    supports_graph_capture = True
    # Phase marks of the step (set by the model runner; a no-op timer by default).
    timer = NULL_TIMER

    def begin_step(self, stage_tokens: dict[int, int], **flags: Any) -> None:
        """``flags``: is_warmup / is_graph_capturing / is_graph_replaying / tokens_across_attn."""
        return None

    def step_prologue(self) -> None:
        """Device work issued at the start of every forward (inside captured graphs)."""
        return None

    def send(self, layer_idx: int, attn_out: torch.Tensor, residual: torch.Tensor, stage_idx: int) -> Any:
        raise NotImplementedError

    def recv(self, layer_idx: int, handle: Any, stage_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        raise NotImplementedError

    def end_step(self) -> None:
        return None


class LocalFFNExecutor(FFNExecutor):
    def __init__(self, model):
        self.model = model

    def send(self, layer_idx, attn_out, residual, stage_idx):
        h, residual = self.model.post_attention_norm(layer_idx, attn_out, residual)
        return self.model.compute_ffn_output(h, layer_idx, **self.model.ffn_extra(layer_idx, residual)), residual

    def recv(self, layer_idx, handle, stage_idx):
        return handle


@dataclass
class _Pending:
    ref: torch.Tensor
    residual: torch.Tensor
    local_out: torch.Tensor | None = None


class ConnectorFFNExecutor(FFNExecutor):
    """Sends post-norm hidden states through ``connector`` and receives the FFN output.

    ``attn_dp_group`` is a (gloo) group over all Attention ranks used to
    exchange per-stage token counts each step, the information vLLM's DP
    metadata carries in the reference.
    """

    @property
    def supports_graph_capture(self) -> bool:
        """Decode graphs need stream-ordered transfers (the NCCL connector's subgroup
        communicator on GPUs); asked of the connector once it is initialised."""
        return bool(getattr(self.connector, "supports_graph_capture", False))

    def __init__(self, model, connector, *, attn_dp_group=None, attn_size: int = 1, attn_rank: int = 0):
        self.model = model
        self.connector = connector
        self.group = attn_dp_group
        self.attn_size = attn_size
        self.attn_rank = attn_rank
        self.gate_on_attn = model.compute_gate_on_attention

    def begin_step(self, stage_tokens, *, is_warmup=False, is_graph_capturing=False, is_graph_replaying=False,
                   tokens_across_attn: dict[int, tuple[int, ...]] | None = None):
        stages = sorted(stage_tokens)
        if tokens_across_attn is not None:
            table = torch.tensor([[max(1, int(tokens_across_attn[s][a])) for s in stages]
                                  for a in range(self.attn_size)], dtype=torch.int32)
        elif self.group is not None and self.attn_size > 1:
            local = torch.tensor([max(1, int(stage_tokens[s])) for s in stages], dtype=torch.int32)
            gathered = [torch.empty_like(local) for _ in range(self.attn_size)]
            dist.all_gather(gathered, local, group=self.group)
            table = torch.stack(gathered)  # [A, stages]
        else:
            table = torch.tensor([[max(1, int(stage_tokens[s])) for s in stages]], dtype=torch.int32)
        payload = AFDControlPayload(
            dp_metadata_list={s: AFDDPMetadata(num_tokens_across_dp_cpu=table[:, i].clone())
                              for i, s in enumerate(stages)},
            is_graph_capturing=is_graph_capturing,
            is_warmup=is_warmup,
            is_graph_replaying=is_graph_replaying,
        )
        cp = self.connector.control_plane
        cp.update_state_from_dp_metadata(payload)
        cp.send_dp_metadata_list(payload)

    def send(self, layer_idx, attn_out, residual, stage_idx):
        model = self.model
        h, residual = model.post_attention_norm(layer_idx, attn_out, residual)
        is_moe = model.arch.is_moe_layer(layer_idx)
        if self.gate_on_attn and not is_moe:
            # Dense layers stay on the Attention side when the gate does.
            return _Pending(ref=h, residual=residual, local_out=model.compute_ffn_output(h, layer_idx))
        ctx = AFDTransferContext(
            metadata=AFDTransferMetadata.create_attention_metadata(
                layer_idx=layer_idx, stage_idx=stage_idx, seq_len=int(h.shape[0]))
        )
        kwargs = dict(model.ffn_extra(layer_idx, residual))
        if "input_ids" in kwargs:
            kwargs["input_ids"] = kwargs["input_ids"].to(torch.int32)
        if self.gate_on_attn:
            kwargs["router_logits"] = model.compute_router_logits(layer_idx, h)
        self.connector.send_attn_output(h, ctx, **kwargs)
        return _Pending(ref=torch.empty_like(h), residual=residual)

    def recv(self, layer_idx, handle: _Pending, stage_idx):
        if handle.local_out is not None:
            return handle.local_out, handle.residual
        out = self.connector.recv_ffn_output(ref_tensor=handle.ref, ubatch_idx=stage_idx)
        return out, handle.residual

    def shutdown_remote(self) -> None:
        """Tell the FFN loop to exit (control-plane senders only)."""
        payload = AFDControlPayload(dp_metadata_list={0: AFDDPMetadata(num_tokens_across_dp_cpu=[1])},
                                    is_graph_capturing=False, is_warmup=False, is_shutdown=True)
        self.connector.control_plane.send_dp_metadata_list(payload)


__all__ = ["ConnectorFFNExecutor", "FFNExecutor", "LocalFFNExecutor"]
