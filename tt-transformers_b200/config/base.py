"""Helpers for reading typed values out of a config.json dictionary."""

from __future__ import annotations

import json
import os


class ConfigError(ValueError):
    """A config.json key is missing, has the wrong type or an unsupported value."""


_MISSING = object()


def read_config_json(folder: str) -> dict:
    path = os.path.join(folder, "config.json")
    if not os.path.isfile(path):
        raise ConfigError(f"{folder}: no config.json")
    with open(path) as f:
        data = json.load(f)
    if not isinstance(data, dict):
        raise ConfigError(f"{path}: top level must be an object")
    return data


def take(data: dict, key: str, kind, default=_MISSING, *, where: str = "config.json"):
    """data[key] converted to `kind` (int, float, bool, str); ConfigError names the key."""
    value = data.get(key, None)
    if value is None:
        if default is _MISSING:
            raise ConfigError(f"{where}: required key '{key}' is missing")
        return default
    if kind is bool:
        if not isinstance(value, bool):
            raise ConfigError(f"{where}: '{key}' must be true or false, got {value!r}")
        return value
    if kind is int:
        if isinstance(value, bool) or not isinstance(value, int):
            if isinstance(value, float) and value == int(value):
                return int(value)
            raise ConfigError(f"{where}: '{key}' must be an integer, got {value!r}")
        return value
    if kind is float:
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise ConfigError(f"{where}: '{key}' must be a number, got {value!r}")
        return float(value)
    if kind is str:
        if not isinstance(value, str):
            raise ConfigError(f"{where}: '{key}' must be a string, got {value!r}")
        return value
    raise TypeError(kind)


def require(condition: bool, message: str) -> None:
    if not condition:
        raise ConfigError(message)
