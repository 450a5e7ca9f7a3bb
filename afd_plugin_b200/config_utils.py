"""Strict scalar coercion for AFD configuration values.

Behavioural parity with ``afd_plugin/config_utils.py:8-75`` of the reference:
booleans accept bool / 0 / 1 / common yes-no strings, integers refuse floats
and bools, positive integers reject zero and negatives.
"""

from __future__ import annotations

_TRUE_WORDS = frozenset({"1", "true", "yes", "on"})
_FALSE_WORDS = frozenset({"0", "false", "no", "off"})


def coerce_extra_bool(value: object, *, field_name: str) -> bool:
    """Return ``value`` as a bool, or raise ``TypeError`` naming ``field_name``."""
    if isinstance(value, bool):
        return value
    if isinstance(value, int) and value in (0, 1):
        return bool(value)
    if isinstance(value, str):
        word = value.strip().lower()
        if word in _TRUE_WORDS:
            return True
        if word in _FALSE_WORDS:
            return False
    raise TypeError(f"{field_name} must be a boolean, got {value!r}")


def coerce_extra_str(value: object, *, field_name: str) -> str:
    """Return a stripped lower-case string, or raise ``TypeError``."""
    if not isinstance(value, str):
        raise TypeError(f"{field_name} must be a string, got {value!r}")
    return value.strip().lower()


def coerce_extra_int(value: object, *, field_name: str) -> int:
    """Return ``value`` as an int without silently truncating floats."""
    if isinstance(value, (bool, float)):
        raise TypeError(f"{field_name} must be an integer, got {value!r}")
    try:
        return int(value)  # type: ignore[arg-type]
    except (TypeError, ValueError, OverflowError) as exc:
        raise TypeError(f"{field_name} must be an integer, got {value!r}") from exc


def coerce_extra_positive_int(value: object, *, field_name: str) -> int:
    """Return a strictly positive int, or raise."""
    number = coerce_extra_int(value, field_name=field_name)
    if number <= 0:
        raise ValueError(f"{field_name} must be positive, got {number}")
    return number


def coerce_optional_extra_positive_int(value: object, *, field_name: str) -> int | None:
    """Like :func:`coerce_extra_positive_int` but ``None``/``""`` map to ``None``."""
    if value is None or value == "":
        return None
    return coerce_extra_positive_int(value, field_name=field_name)


__all__ = [
    "coerce_extra_bool",
    "coerce_extra_int",
    "coerce_extra_positive_int",
    "coerce_extra_str",
    "coerce_optional_extra_positive_int",
]
