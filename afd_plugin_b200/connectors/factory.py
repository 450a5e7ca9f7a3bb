"""Name -> connector class registry with lazy imports.

Mirrors ``AFDConnectorFactory`` of the reference (``connectors/factory.py:23-85``).
The Ascend connector names are registered as refusals so a shared config
produces a clear error on B200 instead of an unknown-name failure.
"""

from __future__ import annotations

import importlib
from typing import Any

from afd_plugin_b200.config import AFDConfig
from afd_plugin_b200.connectors.base import AFDConnectorBase

_NPU_ONLY = {
    "CAMP2pAFDConnector": "Ascend NPU HCCL-window connector",
    "CAMAsyncAFDConnector": "Ascend NPU closed CAM async connector",
}


class AFDConnectorFactory:
    _registry: dict[str, tuple[str, str]] = {}

    @classmethod
    def register_connector(cls, name: str, module: str, class_name: str) -> None:
        if name in cls._registry:
            raise ValueError(f"AFD connector {name!r} is already registered")
        cls._registry[name] = (module, class_name)

    @classmethod
    def registered(cls) -> tuple[str, ...]:
        return tuple(cls._registry)

    @classmethod
    def get_connector_class(cls, name: str) -> type[AFDConnectorBase]:
        if name in _NPU_ONLY:
            raise RuntimeError(f"{name} is an {_NPU_ONLY[name]} and is not available on B200")
        if name not in cls._registry:
            raise ValueError(f"unsupported AFD connector {name!r}; registered: {sorted(cls._registry)}")
        module, class_name = cls._registry[name]
        return getattr(importlib.import_module(module), class_name)

    @classmethod
    def create_connector(
        cls, rank: int, local_rank: int, engine_config: Any, afd_config: AFDConfig, role_rank: int | None = None
    ) -> AFDConnectorBase:
        if role_rank is None:
            from afd_plugin_b200.parallel.topology import resolve_role_rank

            role_rank = resolve_role_rank(engine_config.parallel_config, afd_config)
        klass = cls.get_connector_class(afd_config.connector)
        return klass(rank, local_rank, engine_config, afd_config, role_rank)


AFDConnectorFactory.register_connector(
    "P2pNcclAFDConnector", "afd_plugin_b200.connectors.p2p_nccl", "P2pNcclAFDConnector"
)
AFDConnectorFactory.register_connector(
    "B200FusedAFDConnector", "afd_plugin_b200.connectors.b200_fused", "B200FusedAFDConnector"
)

__all__ = ["AFDConnectorFactory"]
