"""Point-to-point AFD connector with the reference's wire semantics.

This is the baseline the fused B200 connector is measured against, and the
transport of the CPU/gloo multi-rank tests.  Behaviour follows
``P2pNcclAFDConnector`` (``afd_plugin/connectors/gpu/p2p.py:114-888``):

* world order ``[F..., A...]`` and one subgroup per FFN rank;
* Attention sends ``[T, H]`` hidden states (then router logits when the gate
  runs on Attention, then ``int32`` input ids when the model needs them) to its
  FFN rank; the FFN rank receives from every subgroup peer in order,
  concatenates, computes, splits the output by the recorded sequence lengths
  and sends each slice back;
* zero-token peers are clamped to one placeholder row;
* a control plane carries per-stage DP token counts (JSON codec) from the
  first ``min(A, F)`` Attention ranks to the FFN ranks.

Transport: on GPUs one NCCL communicator per subgroup (created from a unique
id the FFN rank shares over a gloo group, as the reference builds a
``PyNcclCommunicator`` per subgroup, ``p2p.py:269-286``), with ``ncclSend`` /
``ncclRecv`` issued on the caller's current stream -- so a decode step
through this connector captures into a CUDA graph on both roles, like the
reference's graph-capturable custom ops (``p2p.py:905-992``).  On CPU,
``torch.distributed`` point-to-point over gloo.  The control payload travels
over a gloo group on host tensors, so the FFN side never synchronises the
device to read it (the reference stages it on the GPU and pays a
``.item()`` sync).
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any, NamedTuple

import torch
import torch.distributed as dist

from afd_plugin_b200.config import AFDConfig
from afd_plugin_b200.connectors.base import AFDConnectorBase, AFDControlPlane, ConnectorExtraInfo
from afd_plugin_b200.connectors.metadata import (
    AFDA2FTransferPayload,
    AFDControlPayload,
    AFDDPMetadata,
    AFDExpertRoutingSpec,
    AFDTransferContext,
    AFDTransferMetadata,
    recv_control_payload,
    send_control_payload,
)
from afd_plugin_b200.parallel.topology import build_rank_mapping

_INPUT_IDS_DTYPE = torch.int32


class _WireSpec(NamedTuple):
    device: torch.device
    dtype: torch.dtype
    size: torch.Size


def init_subgroup_comm(mapping, *, attention_size: int, ffn_size: int, device) -> int:
    """One NCCL communicator per FFN subgroup (the FFN rank first, then its
    Attention ranks); returns this rank's communicator handle.  Every world
    rank takes part in creating every subgroup's gloo group (a collective),
    then joins its own communicator; its send/recv run on the caller's
    current stream, so they can be captured into a CUDA graph."""
    from afd_plugin_b200.ops._ext import ops

    C = ops()
    F, r = ffn_size, attention_size // ffn_size
    mine = None
    for k in range(F):
        members = [k] + [F + k * r + j for j in range(r)]
        g = dist.new_group(ranks=members, backend="gloo")
        if k == mapping.subgroup_index:
            mine = (g, members)
    g, members = mine
    box = [C.nccl_unique_id() if mapping.rank_in_subgroup == 0 else None]
    dist.broadcast_object_list(box, src=members[0], group=g)
    torch.cuda.set_device(device)
    return int(C.nccl_comm_init(box[0], len(members), mapping.rank_in_subgroup))


def num_tokens_for_attention_rank(dp_metadata: AFDDPMetadata, *, attention_rank: int, attention_size: int,
                                  fallback: int = 1) -> int:
    """Tokens one Attention rank puts on the wire for a stage (never below one)."""
    counts = dp_metadata.num_tokens_across_dp_cpu.flatten().tolist()
    if not counts:
        return max(1, fallback)
    if len(counts) < attention_size and attention_size % len(counts) == 0:
        tp = attention_size // len(counts)
        counts = [counts[i // tp] for i in range(attention_size)]
    if 0 <= attention_rank < len(counts):
        return max(1, int(counts[attention_rank]))
    return max(1, fallback)


class P2pNcclAFDConnector(AFDConnectorBase):
    """Reference-semantics send/recv connector (NCCL on CUDA, gloo on CPU)."""

    @classmethod
    def parse_extra_config(cls, raw: Mapping[str, Any] | None) -> ConnectorExtraInfo:
        if raw is not None and not isinstance(raw, Mapping):
            raise TypeError("P2P connector_extra_config must be a mapping")
        if raw:
            raise ValueError("P2pNcclAFDConnector does not support connector_extra_config")
        return ConnectorExtraInfo()

    def __init__(self, rank: int, local_rank: int, engine_config: Any, afd_config: AFDConfig, role_rank: int) -> None:
        super().__init__(rank, local_rank, engine_config, afd_config, role_rank)
        self._initialized = False
        self.mapping = build_rank_mapping(afd_config, role_rank)
        self.world_rank = self.mapping.world_rank
        self.p2p_rank = self.mapping.p2p_rank
        self.attn_size = self.mapping.attention_size
        self.ffn_size = self.mapping.ffn_size
        self.min_size = self.mapping.min_size
        self.ratio = self.mapping.ratio
        self.group_size = len(self.mapping.subgroup_ranks)
        self.dst_list = list(self.mapping.dp_metadata_destinations)
        arch = engine_config.model_config.hf_config
        self.hidden_size = arch.hidden_size
        self.dtype = engine_config.model_config.dtype
        self.device = torch.device("cuda", local_rank) if torch.cuda.is_available() and self._use_cuda() else torch.device("cpu")
        self.dp_metadata_list: dict[int, AFDDPMetadata] = {}
        self.is_graph_capturing = False
        self.is_warmup = False
        self.tensor_metadata_list: dict[int, _WireSpec] = {}
        self._peer_specs: dict[tuple[int, int], _WireSpec] = {}
        self._recv_buffers: dict[tuple[int, int, tuple[int, ...]], torch.Tensor] = {}
        self._ids_buffers: dict[tuple[int, int, tuple[int, ...]], torch.Tensor] = {}
        self.control_group = None
        # In-flight sends: (work, tensor kept alive until the work completes).
        self._pending: list[tuple[object, torch.Tensor]] = []
        self._comm = 0  # NCCL communicator of this rank's subgroup (GPU transport)
        self.control_plane = P2pNcclAFDControlPlane(self)

    @property
    def supports_graph_capture(self) -> bool:
        """Stream-ordered NCCL sends / receives capture into decode graphs."""
        return bool(self._comm)

    def _use_cuda(self) -> bool:
        return dist.is_initialized() and dist.get_backend() == "nccl"

    # --------------------------------------------------------- lifecycle
    def init_afd_connector(self) -> None:
        """Collective over the AFD world: every rank builds the same groups."""
        if self._initialized:
            return
        if not dist.is_initialized():
            raise RuntimeError("P2pNcclAFDConnector needs the AFD world (torch.distributed) initialised")
        if dist.get_world_size() != self.attn_size + self.ffn_size:
            raise RuntimeError(
                f"AFD world has {dist.get_world_size()} ranks, config expects {self.attn_size + self.ffn_size}"
            )
        if dist.get_rank() != self.world_rank:
            raise RuntimeError(f"process has world rank {dist.get_rank()}, AFD topology expects {self.world_rank}")
        control_ranks = list(range(self.ffn_size + self.min_size))
        group = dist.new_group(ranks=control_ranks, backend="gloo")
        self.control_group = group if self.mapping.participates_in_dp_metadata_group else None
        # Two ubatches keep torch.distributed's asynchronous sends: with stream-ordered
        # sends, a rank's second send would queue ahead of its first receive.
        ubatching = bool(getattr(getattr(self.engine_config, "parallel_config", None), "use_ubatching", False))
        if self.device.type == "cuda" and self.group_size > 1 and not ubatching:
            self._comm = self._init_subgroup_comm()
        self._initialized = True

    def _init_subgroup_comm(self) -> int:
        return init_subgroup_comm(self.mapping, attention_size=self.attn_size, ffn_size=self.ffn_size,
                                  device=self.device)

    def close(self) -> None:
        self.flush()
        if self._comm:
            torch.cuda.synchronize(self.device)
            from afd_plugin_b200.ops._ext import ops

            ops().nccl_comm_destroy(self._comm)
            self._comm = 0
        self.control_group = None
        self._recv_buffers.clear()
        self._ids_buffers.clear()
        self._initialized = False

    @property
    def is_initialized(self) -> bool:
        return self._initialized

    # ----------------------------------------------------------- helpers
    def _peer(self, subgroup_rank: int) -> int:
        return self.mapping.subgroup_ranks[subgroup_rank]

    def _send(self, t: torch.Tensor, subgroup_dst: int) -> None:
        if not self._initialized:
            raise RuntimeError("P2P connector is not initialized")
        if self.group_size == 1:
            return
        if subgroup_dst >= self.group_size:
            raise ValueError(f"invalid P2P destination rank {subgroup_dst}")
        if self.device.type == "cuda" and not t.is_cuda:
            raise ValueError("P2P hidden states must be on GPU")
        t = t.contiguous()
        if self._comm:
            # stream-ordered: the buffer stays valid until the send completes (the
            # caching allocator reuses it only behind this stream's later work)
            torch.ops.afd_b200.nccl_send(t, subgroup_dst, self._comm)
            return
        # Sends are posted without blocking so that, under DBO, a rank can post
        # its next ubatch's send before it receives the previous one's result.
        self._pending.append((dist.isend(t, dst=self._peer(subgroup_dst)), t))

    def flush(self) -> None:
        """Wait for every posted send (end of step, or before buffers are reused)."""
        pending, self._pending = self._pending, []
        for work, _ in pending:
            work.wait()

    def _recv(self, subgroup_src: int, spec: _WireSpec, ref_tensor: torch.Tensor | None = None) -> torch.Tensor:
        if not self._initialized:
            raise RuntimeError("P2P connector is not initialized")
        if self.group_size == 1:
            if ref_tensor is None:
                raise RuntimeError("single-rank P2P recv requires a reference tensor")
            return ref_tensor
        size = list(spec.size)
        if ref_tensor is not None:
            size[0] = ref_tensor.shape[0]
        if (ref_tensor is not None and tuple(ref_tensor.shape) == tuple(size)
                and ref_tensor.dtype == spec.dtype and ref_tensor.device == spec.device):
            out = ref_tensor
        else:
            out = torch.empty(size, dtype=spec.dtype, device=spec.device)
        if self._comm:
            torch.ops.afd_b200.nccl_recv(out, subgroup_src, self._comm)
        else:
            dist.recv(out, src=self._peer(subgroup_src))
        return out

    # ---------------------------------------------------- attention side
    def send_attn_output(self, hidden_states: torch.Tensor, context: AFDTransferContext, **kwargs: Any) -> None:
        meta = context.metadata
        if not meta.validate_tensor_shape(tuple(hidden_states.shape)):
            raise ValueError(
                f"hidden_states shape {tuple(hidden_states.shape)!r} does not match AFD metadata token count "
                f"{meta.total_tokens}"
            )
        router_logits = kwargs.get("router_logits")
        input_ids = kwargs.get("input_ids")
        if router_logits is not None and router_logits.shape[0] != hidden_states.shape[0]:
            raise ValueError("router_logits and hidden_states must have equal token counts")
        if input_ids is not None:
            if input_ids.ndim != 1 or input_ids.shape[0] != hidden_states.shape[0]:
                raise ValueError("input_ids must be one-dimensional and token-aligned with hidden_states")
            if input_ids.dtype != _INPUT_IDS_DTYPE:
                raise ValueError("P2P AFD input_ids must use torch.int32")
        self._send(hidden_states, 0)
        if router_logits is not None:
            self._send(router_logits, 0)
        if input_ids is not None:
            self._send(input_ids, 0)

    def recv_ffn_output(self, ref_tensor: torch.Tensor, ubatch_idx: int = 0, **kwargs: Any) -> torch.Tensor:
        out = self._recv(0, self.tensor_metadata_list[ubatch_idx], ref_tensor=ref_tensor)
        self.flush()
        return out

    # ---------------------------------------------------------- FFN side
    def recv_attn_output(self, ubatch_idx: int = 0, **kwargs: Any) -> AFDA2FTransferPayload:
        routing_spec: AFDExpertRoutingSpec | None = kwargs.get("routing_spec")
        want_ids: bool = kwargs.get("recv_input_ids", False)
        graphs = not self.engine_config.model_config.enforce_eager
        hidden, logits, ids = [], [], []
        for src in range(1, self.group_size):
            spec = self._peer_specs.get((ubatch_idx, src), self.tensor_metadata_list[ubatch_idx])
            buf = self._recv_buffers.get((ubatch_idx, src, tuple(spec.size))) if graphs else None
            hidden.append(self._recv(src, spec, ref_tensor=buf))
            if routing_spec is not None:
                lspec = _WireSpec(spec.device, routing_spec.router_logits_dtype,
                                  torch.Size([spec.size[0], routing_spec.router_logits_width]))
                logits.append(self._recv(src, lspec))
            if want_ids:
                ispec = _WireSpec(spec.device, _INPUT_IDS_DTYPE, torch.Size([spec.size[0]]))
                ibuf = self._ids_buffers.get((ubatch_idx, src, (spec.size[0],))) if graphs else None
                ids.append(self._recv(src, ispec, ref_tensor=ibuf))
        if not hidden:
            raise RuntimeError("P2P FFN rank has no Attention peers")
        self.flush()

        def cat(xs):
            return xs[0] if len(xs) == 1 else torch.cat(xs, dim=0)

        meta = AFDTransferMetadata.create_ffn_metadata(
            layer_idx=0, stage_idx=ubatch_idx, seq_lens=[t.shape[0] for t in hidden]
        )
        return AFDA2FTransferPayload(
            hidden_states=cat(hidden),
            context=AFDTransferContext(metadata=meta),
            router_logits=cat(logits) if logits else None,
            input_ids=cat(ids) if ids else None,
        )

    def send_ffn_output(self, ffn_output: torch.Tensor, context: AFDTransferContext, **kwargs: Any) -> None:
        meta = context.metadata
        if not meta.validate_tensor_shape(tuple(ffn_output.shape)):
            raise ValueError(f"ffn_output shape {tuple(ffn_output.shape)!r} does not match metadata")
        if self.ratio == 1:
            self._send(ffn_output, 1)
            return
        sizes = list(meta.seq_lens)
        if len(sizes) != self.ratio:
            total = ffn_output.shape[0]
            if total % self.ratio:
                raise ValueError(
                    f"cannot evenly split FFN output across Attention peers: tokens={total}, ratio={self.ratio}"
                )
            sizes = [total // self.ratio] * self.ratio
        start = 0
        for dst, n in zip(range(1, self.group_size), sizes):
            self._send(ffn_output[start : start + n], dst)
            start += n


class P2pNcclAFDControlPlane(AFDControlPlane):
    """Control payloads over a gloo group; shapes derived per stage."""

    def __init__(self, connector: P2pNcclAFDConnector) -> None:
        self.connector = connector

    def update_state_from_dp_metadata(self, payload: AFDControlPayload) -> None:
        c = self.connector
        c.dp_metadata_list = payload.dp_metadata_list
        c.is_graph_capturing = payload.is_graph_capturing
        c.is_warmup = payload.is_warmup
        c.tensor_metadata_list = {}
        c._peer_specs = {}
        for stage, dpm in payload.dp_metadata_list.items():
            if c.afd_config.role == "ffn":
                total = 0
                for src in range(1, c.group_size):
                    arank = c.mapping.subgroup_index * c.ratio + src - 1
                    n = num_tokens_for_attention_rank(dpm, attention_rank=arank, attention_size=c.attn_size)
                    c._peer_specs[(stage, src)] = _WireSpec(c.device, c.dtype, torch.Size([n, c.hidden_size]))
                    total += n
            else:
                total = num_tokens_for_attention_rank(dpm, attention_rank=c.mapping.role_rank,
                                                      attention_size=c.attn_size)
            c.tensor_metadata_list[stage] = _WireSpec(c.device, c.dtype, torch.Size([total, c.hidden_size]))
        if c.afd_config.role == "ffn" and not c.engine_config.model_config.enforce_eager:
            for (stage, src), spec in c._peer_specs.items():
                key = (stage, src, tuple(spec.size))
                if key not in c._recv_buffers:
                    c._recv_buffers[key] = torch.empty(tuple(spec.size), dtype=spec.dtype, device=spec.device)
                ikey = (stage, src, (spec.size[0],))
                if ikey not in c._ids_buffers:
                    c._ids_buffers[ikey] = torch.empty((spec.size[0],), dtype=_INPUT_IDS_DTYPE, device=spec.device)

    def send_dp_metadata_list(self, payload: AFDControlPayload) -> None:
        c = self.connector
        if c.control_group is None or not c.mapping.is_attention_top_min_size_rank:
            return
        send_control_payload(payload, dst=c.dst_list, group=c.control_group, device=torch.device("cpu"))

    def recv_dp_metadata_list(self) -> AFDControlPayload:
        c = self.connector
        if c.control_group is None:
            raise RuntimeError("P2P DP metadata process group is not initialized")
        return recv_control_payload(src=c.mapping.control_source(), group=c.control_group, device=torch.device("cpu"))


__all__ = ["P2pNcclAFDConnector", "P2pNcclAFDControlPlane", "init_subgroup_comm", "num_tokens_for_attention_rank"]
