"""AFD connectors: contract, metadata, factory and implementations."""

from afd_plugin_b200.connectors.base import AFDConnectorBase, AFDControlPlane, ConnectorExtraInfo
from afd_plugin_b200.connectors.factory import AFDConnectorFactory
from afd_plugin_b200.connectors.metadata import (
    AFDA2FTransferPayload,
    AFDControlPayload,
    AFDDPMetadata,
    AFDExpertRoutingSpec,
    AFDTransferContext,
    AFDTransferMetadata,
)

__all__ = [
    "AFDA2FTransferPayload",
    "AFDConnectorBase",
    "AFDConnectorFactory",
    "AFDControlPayload",
    "AFDControlPlane",
    "AFDDPMetadata",
    "AFDExpertRoutingSpec",
    "AFDTransferContext",
    "AFDTransferMetadata",
    "ConnectorExtraInfo",
]
