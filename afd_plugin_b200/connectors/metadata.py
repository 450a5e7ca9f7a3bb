"""Metadata objects exchanged between the Attention and FFN roles.

Field names and meanings follow the reference contract
(``afd_plugin/connectors/metadata.py:23-420``) because model wrappers and
runners are written against them; the implementations here carry no vLLM
dependency.  The control payload codec uses the same compact JSON schema
(size message + UTF-8 blob) so a control-plane capture from either stack
decodes in the other.
"""

from __future__ import annotations

import copy
import json
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, NamedTuple

import torch

if TYPE_CHECKING:  # pragma: no cover
    from afd_plugin_b200.connectors.base import AFDConnectorBase


def _as_cpu_i32(value: Any) -> torch.Tensor:
    return torch.as_tensor(value, dtype=torch.int32, device="cpu")


@dataclass(slots=True)
class AFDDPMetadata:
    """Per-data-parallel-rank token counts for one stage (ubatch)."""

    num_tokens_across_dp_cpu: torch.Tensor
    max_tokens_across_dp_cpu: torch.Tensor | None = None
    local_sizes: list[int] | None = None

    def __post_init__(self) -> None:
        self.num_tokens_across_dp_cpu = _as_cpu_i32(self.num_tokens_across_dp_cpu)
        if self.max_tokens_across_dp_cpu is None:
            self.max_tokens_across_dp_cpu = self.num_tokens_across_dp_cpu.max()
        else:
            self.max_tokens_across_dp_cpu = _as_cpu_i32(self.max_tokens_across_dp_cpu)

    def _per_sp_rank(self, sp_size: int) -> torch.Tensor:
        counts = self.num_tokens_across_dp_cpu
        return ((counts + sp_size - 1) // sp_size).repeat_interleave(sp_size)

    @contextmanager
    def sp_local_sizes(self, sequence_parallel_size: int) -> Iterator[list[int]]:
        self.local_sizes = self._per_sp_rank(sequence_parallel_size).tolist()
        try:
            yield self.local_sizes
        finally:
            self.local_sizes = None

    def get_chunk_sizes_across_dp_rank(self) -> list[int] | None:
        return self.local_sizes

    def cu_tokens_across_sp(self, sp_size: int) -> torch.Tensor:
        return torch.cumsum(self._per_sp_rank(sp_size), dim=0)

    @contextmanager
    def chunked_sizes(
        self, sequence_parallel_size: int, max_chunk_size_per_rank: int, chunk_idx: int
    ) -> Iterator[list[int]]:
        per_rank = self._per_sp_rank(sequence_parallel_size).tolist()
        offset = max_chunk_size_per_rank * chunk_idx
        self.local_sizes = [max(1, min(max_chunk_size_per_rank, n - offset)) for n in per_rank]
        try:
            yield self.local_sizes
        finally:
            self.local_sizes = None


AFDSingleDPMetadata = AFDDPMetadata


@dataclass(slots=True)
class AFDControlPayload:
    """Per-step control message: stage -> DP token counts plus mode flags."""

    dp_metadata_list: dict[int, AFDDPMetadata]
    is_graph_capturing: bool
    is_warmup: bool
    is_graph_replaying: bool = False
    is_profile: bool = False
    # Framework extension (ignored by the reference codec): ask the FFN loop to exit.
    is_shutdown: bool = False

    def __post_init__(self) -> None:
        normalised: dict[int, AFDDPMetadata] = {}
        for stage, meta in self.dp_metadata_list.items():
            if not isinstance(meta, AFDDPMetadata):
                meta = AFDDPMetadata(num_tokens_across_dp_cpu=meta.num_tokens_across_dp_cpu)
            normalised[int(stage)] = meta
        self.dp_metadata_list = normalised


@dataclass(slots=True)
class AFDTransferState:
    """Backend-specific per-transfer state (subclassed by connectors)."""


class AFDExpertRoutingSpec(NamedTuple):
    router_logits_width: int
    router_logits_dtype: torch.dtype


@dataclass(slots=True)
class AFDTransferMetadata:
    layer_idx: int
    stage_idx: int
    seq_lens: list[int]

    def __post_init__(self) -> None:
        if not self.seq_lens:
            raise ValueError("seq_lens cannot be empty")
        if any(n <= 0 for n in self.seq_lens):
            raise ValueError("all sequence lengths must be positive")

    @property
    def total_tokens(self) -> int:
        return sum(self.seq_lens)

    @classmethod
    def create_attention_metadata(cls, *, layer_idx: int, stage_idx: int, seq_len: int) -> AFDTransferMetadata:
        return cls(layer_idx=layer_idx, stage_idx=stage_idx, seq_lens=[seq_len])

    @classmethod
    def create_ffn_metadata(cls, *, layer_idx: int, stage_idx: int, seq_lens: list[int]) -> AFDTransferMetadata:
        return cls(layer_idx=layer_idx, stage_idx=stage_idx, seq_lens=list(seq_lens))

    def validate_tensor_shape(self, tensor_shape: tuple[int, ...]) -> bool:
        return len(tensor_shape) > 0 and tensor_shape[0] == self.total_tokens


@dataclass(slots=True)
class AFDTransferContext:
    metadata: AFDTransferMetadata
    states: AFDTransferState | None = None


@dataclass(slots=True)
class AFDA2FTransferPayload:
    hidden_states: torch.Tensor
    context: AFDTransferContext
    router_logits: torch.Tensor | None = None
    input_ids: torch.Tensor | None = None


@dataclass(slots=True)
class AFDF2ATransferPayload:
    routed_output: torch.Tensor
    shared_output: torch.Tensor | None = None


@dataclass(slots=True)
class AFDForwardContextMetadata:
    tokens_start_loc: list[int]
    requests_start_loc: list[int]
    stage_idx: int
    connector: "AFDConnectorBase"
    tokens_lens: list[int]
    num_stages: int
    transaction_id: str | None = None
    tokens_unpadded_lens: list[int] = field(default_factory=list)

    def clone(self) -> AFDForwardContextMetadata:
        twin = copy.copy(self)
        twin.tokens_start_loc = list(self.tokens_start_loc)
        twin.requests_start_loc = list(self.requests_start_loc)
        twin.tokens_lens = list(self.tokens_lens)
        twin.tokens_unpadded_lens = list(self.tokens_unpadded_lens)
        return twin


def _scalar(value: Any) -> int:
    return int(value.item()) if hasattr(value, "item") else int(value)


def encode_control_payload(payload: AFDControlPayload) -> bytes:
    stages = {
        str(int(stage)): {
            "num_tokens_across_dp_cpu": meta.num_tokens_across_dp_cpu.tolist(),
            "max_tokens_across_dp_cpu": _scalar(meta.max_tokens_across_dp_cpu),
        }
        for stage, meta in payload.dp_metadata_list.items()
    }
    wire: dict[str, Any] = {
        "dp_metadata_list": stages,
        "is_graph_capturing": bool(payload.is_graph_capturing),
        "is_warmup": bool(payload.is_warmup),
        "is_graph_replaying": bool(payload.is_graph_replaying),
        "is_profile": bool(payload.is_profile),
    }
    if payload.is_shutdown:
        wire["is_shutdown"] = True
    return json.dumps(wire, separators=(",", ":"), sort_keys=True).encode("utf-8")


def decode_control_payload(blob: bytes) -> AFDControlPayload:
    wire = json.loads(blob.decode("utf-8"))
    stages = {
        int(stage): AFDDPMetadata(
            num_tokens_across_dp_cpu=[int(v) for v in meta["num_tokens_across_dp_cpu"]],
            max_tokens_across_dp_cpu=int(meta["max_tokens_across_dp_cpu"]),
        )
        for stage, meta in wire["dp_metadata_list"].items()
    }
    return AFDControlPayload(
        dp_metadata_list=stages,
        is_graph_capturing=bool(wire.get("is_graph_capturing", False)),
        is_warmup=bool(wire.get("is_warmup", False)),
        is_graph_replaying=bool(wire.get("is_graph_replaying", False)),
        is_profile=bool(wire.get("is_profile", False)),
        is_shutdown=bool(wire.get("is_shutdown", False)),
    )


def send_control_payload(payload: AFDControlPayload, *, dst, group, device: torch.device) -> None:
    """Send ``payload`` as a ``long[1]`` size message then a ``uint8`` blob."""
    blob = encode_control_payload(payload)
    body = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(device)
    size = torch.tensor([body.numel()], dtype=torch.long, device=device)
    for d in [dst] if isinstance(dst, int) else list(dst):
        torch.distributed.send(size, dst=d, group=group)
        torch.distributed.send(body, dst=d, group=group)


def recv_control_payload(*, src: int, group, device: torch.device) -> AFDControlPayload:
    size = torch.empty(1, dtype=torch.long, device=device)
    torch.distributed.recv(size, src=src, group=group)
    body = torch.empty(int(size.item()), dtype=torch.uint8, device=device)
    torch.distributed.recv(body, src=src, group=group)
    return decode_control_payload(body.cpu().numpy().tobytes())


__all__ = [
    "AFDA2FTransferPayload",
    "AFDControlPayload",
    "AFDDPMetadata",
    "AFDExpertRoutingSpec",
    "AFDF2ATransferPayload",
    "AFDForwardContextMetadata",
    "AFDSingleDPMetadata",
    "AFDTransferContext",
    "AFDTransferMetadata",
    "AFDTransferState",
    "decode_control_payload",
    "encode_control_payload",
    "recv_control_payload",
    "send_control_payload",
]
