"""AFD connectors: contract, metadata, factory and implementations."""

from afd_plugin_b200.connectors.base import AFDConnectorBase, AFDControlPlane, ConnectorExtraInfo
from afd_plugin_b200.connectors.factory import AFDConnectorFactory
from afd_plugin_b200.connectors.metadata import (
    AFDA2FTransferPayload,
    AFDControlPayload,
    AFDDPMetadata,
    AFDExpertRoutingSpec,
    AFDF2ATransferPayload,
    AFDForwardContextMetadata,
    AFDTransferContext,
    AFDTransferMetadata,
    AFDTransferState,
)

__all__ = [
    "AFDA2FTransferPayload",
    "AFDConnectorBase",
    "AFDConnectorFactory",
    "AFDControlPayload",
    "AFDControlPlane",
    "AFDDPMetadata",
    "AFDExpertRoutingSpec",
    "AFDF2ATransferPayload",
    "AFDForwardContextMetadata",
    "AFDTransferContext",
    "AFDTransferMetadata",
    "AFDTransferState",
    "ConnectorExtraInfo",
]
