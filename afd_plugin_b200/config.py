"""AFD configuration carried in ``additional_config["afd"]``.

The key set, the legacy ``afd_*`` / ``async`` aliases, strict rejection of
unknown keys and the ``connector_extra_config`` escape hatch follow the
reference (``afd_plugin/config.py:29-329``) so that an existing
``--additional-config '{"afd": {...}}'`` string parses identically here.

Connectors accepted by this framework:

* ``P2pNcclAFDConnector`` -- reference wire semantics over NCCL (or gloo on
  CPU) point-to-point; the baseline and the fallback.
* ``B200FusedAFDConnector`` -- the NVLink peer-memory connector whose
  dispatch/combine run inside the fused sm_100a kernels.
* ``CAMP2pAFDConnector`` / ``CAMAsyncAFDConnector`` -- Ascend-only names; they
  parse (so shared configs stay valid) but the factory refuses them on B200.
"""

from __future__ import annotations

import hashlib
from collections.abc import Mapping
from dataclasses import dataclass, fields
from typing import Any, Final, Literal

from afd_plugin_b200.config_utils import coerce_extra_bool, coerce_extra_int

AFD_ADDITIONAL_CONFIG_KEY: Final[str] = "afd"
AFD_ASYNC_CONNECTOR: Final[str] = "CAMAsyncAFDConnector"
P2P_NCCL_CONNECTOR: Final[str] = "P2pNcclAFDConnector"
B200_FUSED_CONNECTOR: Final[str] = "B200FusedAFDConnector"
AFDRole = Literal["attention", "ffn"]

SUPPORTED_AFD_ROLES: Final[tuple[str, ...]] = ("attention", "ffn")
SUPPORTED_AFD_CONNECTORS: Final[tuple[str, ...]] = (
    P2P_NCCL_CONNECTOR,
    B200_FUSED_CONNECTOR,
    "CAMP2pAFDConnector",
    AFD_ASYNC_CONNECTOR,
)
# Connectors whose topology follows the FFN-first subgroup layout.
_SUBGROUP_TOPOLOGY_CONNECTORS: Final[frozenset[str]] = frozenset(
    {P2P_NCCL_CONNECTOR, B200_FUSED_CONNECTOR}
)

_KEY_ALIASES: Final[dict[str, str]] = {
    "afd_connector": "connector",
    "afd_role": "role",
    "afd_port": "port",
    "afd_host": "host",
    "async": "async_dp",
}


@dataclass(frozen=True)
class AFDConfig:
    """Parsed, immutable AFD settings for one process.

    Role ranks are runtime placement, not configuration, and are therefore not
    stored here (same split as the reference).
    """

    connector: str = P2P_NCCL_CONNECTOR
    async_dp: bool = False
    role: AFDRole = "attention"
    port: int = 1239
    host: str = "127.0.0.1"
    num_attention_ranks: int = 1
    num_ffn_ranks: int = 1
    compute_gate_on_attention: bool = False

    # Legacy read-only spellings.
    @property
    def afd_connector(self) -> str:
        return self.connector

    @property
    def afd_role(self) -> str:
        return self.role

    @property
    def afd_port(self) -> int:
        return self.port

    @property
    def afd_host(self) -> str:
        return self.host

    @property
    def is_attention_server(self) -> bool:
        return self.role == "attention"

    @property
    def is_ffn_server(self) -> bool:
        return self.role == "ffn"

    def compute_hash(self) -> str:
        """Stable digest of the settings that change captured graphs."""
        parts = [
            self.connector,
            self.async_dp,
            self.role,
            self.num_attention_ranks,
            self.num_ffn_ranks,
        ]
        return hashlib.sha256(repr(parts).encode()).hexdigest()

    def validate(self, *, expected_role: str | None = None) -> None:
        validate_afd_config(self, expected_role=expected_role)

    def with_role(self, role: str) -> "AFDConfig":
        """Copy of this config for the other role (used by launchers)."""
        values = {f.name: getattr(self, f.name) for f in fields(self)}
        values["role"] = role
        return AFDConfig(**values)


_FIELD_NAMES: Final[frozenset[str]] = frozenset(f.name for f in fields(AFDConfig))


def _split_raw(raw: Mapping[str, Any]) -> tuple[dict[str, Any], dict[str, Any]]:
    """Canonicalise keys; return ``(afd_fields, connector_extra_config)``."""
    canon: dict[str, Any] = {}
    extra: dict[str, Any] = {}
    for key, value in raw.items():
        name = _KEY_ALIASES.get(key, key)
        if name == "connector_extra_config":
            if not isinstance(value, Mapping):
                raise TypeError(f"{key} must be a mapping")
            extra = dict(value)
            continue
        if name not in _FIELD_NAMES:
            raise ValueError(
                f"unknown AFD config field {key!r}; put connector-specific values "
                "under 'connector_extra_config'"
            )
        if name in canon:
            raise ValueError(
                f"duplicate AFD config field for {name!r}: both alias and canonical "
                "key were provided"
            )
        canon[name] = value

    if "async_dp" in canon:
        canon["async_dp"] = coerce_extra_bool(canon["async_dp"], field_name="async")
    for name in ("port", "num_attention_ranks", "num_ffn_ranks"):
        if name in canon:
            canon[name] = coerce_extra_int(canon[name], field_name=name)
    if "compute_gate_on_attention" in canon:
        canon["compute_gate_on_attention"] = coerce_extra_bool(
            canon["compute_gate_on_attention"], field_name="compute_gate_on_attention"
        )
    return canon, extra


def afd_config_from_mapping(
    raw: Mapping[str, Any], *, validate: bool = True, expected_role: str | None = None
) -> AFDConfig:
    if not isinstance(raw, Mapping):
        raise TypeError(f"AFD config must be a mapping, got {type(raw).__name__}")
    canon, _ = _split_raw(raw)
    cfg = AFDConfig(**canon)
    if validate:
        cfg.validate(expected_role=expected_role)
    return cfg


def connector_extra_config_from_mapping(raw: Mapping[str, Any]) -> dict[str, Any]:
    if not isinstance(raw, Mapping):
        raise TypeError(f"AFD config must be a mapping, got {type(raw).__name__}")
    return _split_raw(raw)[1]


def _additional_config(source: Any) -> Mapping[str, Any] | None:
    if source is None:
        return None
    if isinstance(source, Mapping):
        extra = source
    elif hasattr(source, "additional_config"):
        extra = source.additional_config
    else:
        # a config object without the field is a caller bug, not "AFD off"
        raise AttributeError(f"{type(source).__name__} has no additional_config to read the AFD config from")
    if extra is None:
        return None
    if not isinstance(extra, Mapping):
        raise TypeError(
            "additional_config must be a mapping when parsing AFD config, "
            f"got {type(extra).__name__}"
        )
    return extra


def _afd_section(source: Any) -> Mapping[str, Any] | None:
    extra = _additional_config(source)
    if extra is None or AFD_ADDITIONAL_CONFIG_KEY not in extra:
        return None
    section = extra[AFD_ADDITIONAL_CONFIG_KEY]
    if not isinstance(section, Mapping):
        raise TypeError(f"AFD config must be a mapping, got {type(section).__name__}")
    return section


def has_afd_config(source: Any) -> bool:
    extra = _additional_config(source)
    return extra is not None and AFD_ADDITIONAL_CONFIG_KEY in extra


def parse_optional_afd_config(
    source: Any, *, validate: bool = True, expected_role: str | None = None
) -> AFDConfig | None:
    """Parse ``additional_config["afd"]`` if present, else ``None``."""
    section = _afd_section(source)
    if section is None:
        return None
    return afd_config_from_mapping(section, validate=validate, expected_role=expected_role)


def parse_afd_config(
    source: Any, *, validate: bool = True, expected_role: str | None = None
) -> AFDConfig:
    """Parse the mandatory ``additional_config["afd"]`` section."""
    cfg = parse_optional_afd_config(source, validate=validate, expected_role=expected_role)
    if cfg is None:
        raise ValueError('AFD config requires additional_config["afd"]; omit it to disable AFD')
    return cfg


def connector_extra_config_from_source(source: Any) -> dict[str, Any]:
    section = _afd_section(source)
    if section is None:
        return {}
    return connector_extra_config_from_mapping(section)


def is_afd_active(source: Any) -> bool:
    return parse_optional_afd_config(source, validate=True) is not None


def is_afd_async_dp(source: Any) -> bool:
    cfg = parse_optional_afd_config(source, validate=False)
    return cfg is not None and cfg.async_dp and cfg.connector == AFD_ASYNC_CONNECTOR


def validate_afd_config(cfg: AFDConfig, *, expected_role: str | None = None) -> None:
    """Common AFD validation; imports nothing heavy (safe on CPU-only hosts)."""
    if cfg.role not in SUPPORTED_AFD_ROLES:
        raise ValueError(f"AFD role must be one of {SUPPORTED_AFD_ROLES!r}, got {cfg.role!r}")
    if expected_role is not None and cfg.role != expected_role:
        raise ValueError(f"AFD role mismatch: expected {expected_role!r}, got {cfg.role!r}")
    if cfg.connector not in SUPPORTED_AFD_CONNECTORS:
        raise ValueError(
            f"AFD connector must be one of {SUPPORTED_AFD_CONNECTORS!r}, got {cfg.connector!r}"
        )
    if cfg.async_dp and cfg.connector != AFD_ASYNC_CONNECTOR:
        raise ValueError("AFD async mode requires connector='CAMAsyncAFDConnector'")
    if cfg.connector in _SUBGROUP_TOPOLOGY_CONNECTORS:
        from afd_plugin_b200.parallel.topology import validate_p2p_topology

        validate_p2p_topology(cfg)
    if not cfg.host:
        raise ValueError("AFD host must be non-empty")
    if not 0 < cfg.port < 65536:
        raise ValueError(f"AFD port must be in 1..65535, got {cfg.port}")
    if cfg.num_attention_ranks <= 0:
        raise ValueError(f"num_attention_ranks must be positive, got {cfg.num_attention_ranks}")
    if cfg.num_ffn_ranks <= 0:
        raise ValueError(f"num_ffn_ranks must be positive, got {cfg.num_ffn_ranks}")


__all__ = [
    "AFDConfig",
    "AFDRole",
    "AFD_ADDITIONAL_CONFIG_KEY",
    "AFD_ASYNC_CONNECTOR",
    "B200_FUSED_CONNECTOR",
    "P2P_NCCL_CONNECTOR",
    "SUPPORTED_AFD_CONNECTORS",
    "SUPPORTED_AFD_ROLES",
    "afd_config_from_mapping",
    "connector_extra_config_from_mapping",
    "connector_extra_config_from_source",
    "has_afd_config",
    "is_afd_active",
    "is_afd_async_dp",
    "parse_afd_config",
    "parse_optional_afd_config",
    "validate_afd_config",
]
