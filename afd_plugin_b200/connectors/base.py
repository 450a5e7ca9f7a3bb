"""Connector contract between the Attention and FFN roles.

Method names, arguments and the optional control plane match the reference
interface (``afd_plugin/connectors/base.py:37-307``) so model wrappers and
runners written against it need no change.  Two connectors implement it here:
the NCCL point-to-point baseline and the B200 fused peer-memory connector.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch

from afd_plugin_b200.config import AFDConfig, connector_extra_config_from_source
from afd_plugin_b200.connectors.metadata import AFDA2FTransferPayload, AFDControlPayload, AFDTransferContext


@dataclass(frozen=True)
class ConnectorExtraInfo:
    """Connector-owned options parsed from ``connector_extra_config``."""

    @classmethod
    def from_mapping(cls, raw: Mapping[str, Any] | None) -> "ConnectorExtraInfo":
        raise NotImplementedError

    def to_mapping(self) -> dict[str, Any]:
        return {}


class AFDConnectorBase(ABC):
    """Lifecycle + data path of an AFD connector.

    ``control_plane`` set: FFN steps are driven by control payloads.
    ``control_plane`` ``None``: the connector's own receive loop drives the FFN.
    """

    control_plane: "AFDControlPlane | None" = None
    attn_size: int = 0
    ffn_size: int = 0

    @classmethod
    @abstractmethod
    def parse_extra_config(cls, raw: Mapping[str, Any] | None) -> ConnectorExtraInfo: ...

    def __init__(self, rank: int, local_rank: int, engine_config: Any, afd_config: AFDConfig, role_rank: int) -> None:
        self.rank = rank
        self.local_rank = local_rank
        self.engine_config = engine_config
        self.afd_config = afd_config
        self.role_rank = role_rank
        self.extra_info = self.parse_extra_config(connector_extra_config_from_source(engine_config))

    # reference spelling
    @property
    def vllm_config(self) -> Any:
        return self.engine_config

    @abstractmethod
    def close(self) -> None: ...

    @abstractmethod
    def init_afd_connector(self) -> None: ...

    @property
    @abstractmethod
    def is_initialized(self) -> bool: ...

    # Attention side
    @abstractmethod
    def send_attn_output(self, hidden_states: torch.Tensor, context: AFDTransferContext, **kwargs: Any) -> None: ...

    @abstractmethod
    def recv_ffn_output(self, ref_tensor: torch.Tensor, ubatch_idx: int = 0, **kwargs: Any) -> torch.Tensor: ...

    # FFN side
    @abstractmethod
    def recv_attn_output(self, ubatch_idx: int = 0, **kwargs: Any) -> AFDA2FTransferPayload: ...

    @abstractmethod
    def send_ffn_output(self, ffn_output: torch.Tensor, context: AFDTransferContext, **kwargs: Any) -> None: ...


class AFDControlPlane(ABC):
    """Per-step DP token-count metadata from Attention to FFN."""

    @abstractmethod
    def update_state_from_dp_metadata(self, payload: AFDControlPayload) -> None: ...

    @abstractmethod
    def send_dp_metadata_list(self, payload: AFDControlPayload) -> None: ...

    @abstractmethod
    def recv_dp_metadata_list(self) -> AFDControlPayload: ...


__all__ = ["AFDConnectorBase", "AFDControlPlane", "ConnectorExtraInfo"]
