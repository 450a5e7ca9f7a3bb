"""Messages between the Attention and FFN roles: the per-step control payload and per-transfer context.

The control payload is what the Attention side tells its FFN ranks once per
step: for every stage (DBO ubatch), how many tokens each Attention (DP) rank
contributes, plus the step's mode flags.  It travels as a size message and a
UTF-8 JSON blob; the JSON field names (``dp_metadata_list``,
``num_tokens_across_dp_cpu``, ``max_tokens_across_dp_cpu``,
``is_graph_capturing``, ``is_warmup``, ``is_graph_replaying``, ``is_profile``)
are the reference's wire schema (``afd_plugin/connectors/metadata.py:320-420``),
so a control message captured from either stack decodes in the other.

Per transfer, the connectors exchange the layer, the stage and the token
count(s) of the rows that move (:class:`AFDTransferMetadata`) and hand the FFN
side its input rows with the optional routing inputs
(:class:`AFDA2FTransferPayload`).  The fused connector carries the counts in
device memory instead; these objects serve its Python API only.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Any, NamedTuple

import torch


@dataclass(slots=True)
class AFDDPMetadata:
    """Tokens each Attention (DP) rank contributes to one stage."""

    num_tokens_across_dp_cpu: torch.Tensor
    max_tokens_across_dp_cpu: torch.Tensor | None = None

    def __post_init__(self) -> None:
        counts = torch.as_tensor(self.num_tokens_across_dp_cpu, dtype=torch.int32, device="cpu")
        self.num_tokens_across_dp_cpu = counts
        peak = counts.max() if counts.numel() else torch.tensor(0, dtype=torch.int32)
        self.max_tokens_across_dp_cpu = (peak if self.max_tokens_across_dp_cpu is None else
                                         torch.as_tensor(self.max_tokens_across_dp_cpu, dtype=torch.int32))


@dataclass(slots=True)
class AFDControlPayload:
    """One step's control message: stage -> token counts, plus the step's mode."""

    dp_metadata_list: dict[int, AFDDPMetadata]
    is_graph_capturing: bool
    is_warmup: bool
    is_graph_replaying: bool = False
    is_profile: bool = False
    # This framework's addition (absent from the reference's schema): the FFN loop exits.
    is_shutdown: bool = False

    def __post_init__(self) -> None:
        self.dp_metadata_list = {
            int(stage): meta if isinstance(meta, AFDDPMetadata) else AFDDPMetadata(meta.num_tokens_across_dp_cpu)
            for stage, meta in self.dp_metadata_list.items()
        }


class AFDExpertRoutingSpec(NamedTuple):
    """Width and dtype of the router logits that travel with a layer's rows (gate on the Attention side)."""

    router_logits_width: int
    router_logits_dtype: torch.dtype


@dataclass(slots=True)
class AFDTransferMetadata:
    """Rows of one transfer: a layer and stage, and the token count of each contributing rank."""

    layer_idx: int
    stage_idx: int
    seq_lens: list[int]

    def __post_init__(self) -> None:
        if not self.seq_lens or min(self.seq_lens) <= 0:
            raise ValueError(f"a transfer needs one or more positive token counts, got {self.seq_lens!r}")

    @property
    def total_tokens(self) -> int:
        return sum(self.seq_lens)

    @classmethod
    def create_attention_metadata(cls, *, layer_idx: int, stage_idx: int, seq_len: int) -> AFDTransferMetadata:
        """What one Attention rank sends: its own rows."""
        return cls(layer_idx, stage_idx, [seq_len])

    @classmethod
    def create_ffn_metadata(cls, *, layer_idx: int, stage_idx: int, seq_lens: list[int]) -> AFDTransferMetadata:
        """What an FFN rank received: one count per Attention peer, in peer order."""
        return cls(layer_idx, stage_idx, list(seq_lens))

    def validate_tensor_shape(self, tensor_shape: tuple[int, ...]) -> bool:
        return bool(tensor_shape) and tensor_shape[0] == self.total_tokens


@dataclass(slots=True)
class AFDTransferContext:
    metadata: AFDTransferMetadata


@dataclass(slots=True)
class AFDA2FTransferPayload:
    """An FFN rank's input for one layer and stage."""

    hidden_states: torch.Tensor
    context: AFDTransferContext
    router_logits: torch.Tensor | None = None  # gate on the Attention side
    input_ids: torch.Tensor | None = None  # hash-routed layers (DeepSeek-V4)


def encode_control_payload(payload: AFDControlPayload) -> bytes:
    """Compact, key-sorted JSON of the payload (the wire schema above)."""
    stages = {}
    for stage, meta in payload.dp_metadata_list.items():
        stages[str(stage)] = {"num_tokens_across_dp_cpu": [int(v) for v in meta.num_tokens_across_dp_cpu.tolist()],
                              "max_tokens_across_dp_cpu": int(meta.max_tokens_across_dp_cpu)}
    doc: dict[str, Any] = {"dp_metadata_list": stages}
    for flag in ("is_graph_capturing", "is_warmup", "is_graph_replaying", "is_profile"):
        doc[flag] = bool(getattr(payload, flag))
    if payload.is_shutdown:
        doc["is_shutdown"] = True
    return json.dumps(doc, separators=(",", ":"), sort_keys=True).encode("utf-8")


def decode_control_payload(blob: bytes) -> AFDControlPayload:
    doc = json.loads(blob.decode("utf-8"))
    stages = {int(k): AFDDPMetadata(v["num_tokens_across_dp_cpu"], v["max_tokens_across_dp_cpu"])
              for k, v in doc["dp_metadata_list"].items()}
    flags = {f: bool(doc.get(f, False))
             for f in ("is_graph_capturing", "is_warmup", "is_graph_replaying", "is_profile", "is_shutdown")}
    return AFDControlPayload(stages, **flags)


def send_control_payload(payload: AFDControlPayload, *, dst, group, device: torch.device) -> None:
    """Sends ``payload`` to ``dst`` (a rank or ranks): an int64 byte count, then the bytes."""
    blob = encode_control_payload(payload)
    body = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(device)
    size = torch.tensor([body.numel()], dtype=torch.long, device=device)
    for d in ([dst] if isinstance(dst, int) else dst):
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
    "AFDTransferContext",
    "AFDTransferMetadata",
    "decode_control_payload",
    "encode_control_payload",
    "recv_control_payload",
    "send_control_payload",
]
