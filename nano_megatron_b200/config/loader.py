"""Strict YAML/dict -> :class:`TrainConfig` loading with dotted overrides.

Behaviour of the reference loader (src/nano_megatron/config/loader.py:31-260):
unknown keys are rejected; values are coerced recursively from the dataclass
type hints (unions, tuples, enums, paths); ``--set a.b=v`` values are parsed as
JSON, then as a Python literal, then kept as a string; JSON text is accepted
when PyYAML is missing; ``WORLD_SIZE`` from the environment feeds validation.
"""

from __future__ import annotations

import ast
import dataclasses
import json
import os
import types
import typing
import warnings
from collections.abc import Mapping, Sequence
from enum import Enum
from pathlib import Path
from typing import Any

from .schema import TrainConfig
from .validation import ValidationResult, validate_config


class ConfigLoadError(ValueError):
    """Malformed file, unknown key or uncoercible value."""


class ConfigWarning(UserWarning):
    """Valid but surprising configuration."""


_HINTS: dict[type, dict[str, Any]] = {}


def _hints(cls: type) -> dict[str, Any]:
    if cls not in _HINTS:
        _HINTS[cls] = typing.get_type_hints(cls)
    return _HINTS[cls]


def _build(cls: type, values: Any, path: str):
    if isinstance(values, cls):
        return values
    if not isinstance(values, Mapping):
        raise ConfigLoadError(f"{path} must be a mapping, got {type(values).__name__}")
    names = {f.name for f in dataclasses.fields(cls)}
    unknown = sorted(set(values) - names)
    if unknown:
        raise ConfigLoadError(f"{path} contains unsupported field(s): {', '.join(unknown)}")
    hints = _hints(cls)
    kwargs = {k: _coerce(v, hints[k], f"{path}.{k}") for k, v in values.items()}
    try:
        return cls(**kwargs)
    except (TypeError, ValueError) as error:
        raise ConfigLoadError(f"{path}: {error}") from error


def _coerce(value: Any, hint: Any, path: str) -> Any:
    origin = typing.get_origin(hint)
    args = typing.get_args(hint)
    if origin in (typing.Union, types.UnionType):
        if value is None and type(None) in args:
            return None
        problems = []
        for option in args:
            if option is type(None):
                continue
            try:
                return _coerce(value, option, path)
            except ConfigLoadError as error:
                problems.append(str(error))
        raise ConfigLoadError(f"{path} does not match any supported type: {'; '.join(problems)}")
    if origin is tuple:
        if isinstance(value, (str, bytes)) or not isinstance(value, Sequence):
            raise ConfigLoadError(f"{path} must be a sequence")
        if len(args) == 2 and args[1] is Ellipsis:
            return tuple(_coerce(v, args[0], f"{path}[{i}]") for i, v in enumerate(value))
        if len(value) != len(args):
            raise ConfigLoadError(f"{path} must contain exactly {len(args)} values")
        return tuple(_coerce(v, a, f"{path}[{i}]") for i, (v, a) in enumerate(zip(value, args)))
    if dataclasses.is_dataclass(hint):
        return _build(hint, value, path)
    if isinstance(hint, type) and issubclass(hint, Enum):
        try:
            return hint(value)
        except ValueError as error:
            choices = ", ".join(str(m.value) for m in hint)
            raise ConfigLoadError(f"{path} must be one of: {choices}; got {value!r}") from error
    if hint is Path:
        if not isinstance(value, (str, Path)):
            raise ConfigLoadError(f"{path} must be a filesystem path string")
        return Path(value)
    if hint is bool:
        if not isinstance(value, bool):
            raise ConfigLoadError(f"{path} must be a boolean, got {value!r}")
        return value
    if hint is int:
        if isinstance(value, bool) or not isinstance(value, int):
            raise ConfigLoadError(f"{path} must be an integer, got {value!r}")
        return value
    if hint is float:
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise ConfigLoadError(f"{path} must be a number, got {value!r}")
        return float(value)
    if hint is str:
        if not isinstance(value, str):
            raise ConfigLoadError(f"{path} must be a string, got {value!r}")
        return value
    if hint is Any:
        return value
    raise ConfigLoadError(f"{path} has unsupported schema type {hint!r}")


def config_from_dict(data: Mapping[str, Any]) -> TrainConfig:
    if not isinstance(data, Mapping):
        raise ConfigLoadError(f"top-level configuration must be a mapping, got "
                              f"{type(data).__name__}")
    try:
        return _build(TrainConfig, data, "config")
    except ConfigLoadError:
        raise
    except (TypeError, ValueError) as error:
        raise ConfigLoadError(str(error)) from error


def config_to_dict(config: Any) -> Any:
    """JSON-ready nested dict of a config (enums -> values, paths -> str)."""
    if dataclasses.is_dataclass(config):
        return {f.name: config_to_dict(getattr(config, f.name)) for f in dataclasses.fields(config)}
    if isinstance(config, Enum):
        return config.value
    if isinstance(config, Path):
        return str(config)
    if isinstance(config, (tuple, list)):
        return [config_to_dict(v) for v in config]
    return config


def parse_override_value(text: str) -> Any:
    stripped = text.strip()
    try:
        return json.loads(stripped)
    except json.JSONDecodeError:
        try:
            return ast.literal_eval(stripped)
        except (ValueError, SyntaxError):
            return stripped


def apply_override(config: dict[str, Any], override: str) -> None:
    if "=" not in override:
        raise ConfigLoadError(f"override must use dotted.path=value syntax, got {override!r}")
    dotted, raw = override.split("=", 1)
    keys = dotted.strip().split(".")
    if not keys or any(not k for k in keys):
        raise ConfigLoadError(f"invalid override path {dotted!r}")
    node = config
    for key in keys[:-1]:
        nxt = node.get(key)
        if nxt is None:
            nxt = node[key] = {}
        if not isinstance(nxt, dict):
            raise ConfigLoadError(f"override path {dotted!r} crosses non-mapping key {key!r}")
        node = nxt
    node[keys[-1]] = parse_override_value(raw)


def _read_mapping(source: Path) -> dict[str, Any]:
    try:
        text = source.read_text(encoding="utf-8")
    except OSError as error:
        raise ConfigLoadError(f"could not read configuration {source}: {error}") from error
    try:
        import yaml
    except ImportError:
        try:
            loaded = json.loads(text)
        except json.JSONDecodeError as error:
            raise ConfigLoadError("loading YAML requires PyYAML; install the project "
                                  f"dependencies or provide JSON-compatible YAML ({source})") \
                from error
    else:
        try:
            loaded = yaml.safe_load(text)
        except yaml.YAMLError as error:
            raise ConfigLoadError(f"invalid YAML in {source}: {error}") from error
    loaded = {} if loaded is None else loaded
    if not isinstance(loaded, Mapping):
        raise ConfigLoadError(f"top-level configuration in {source} must be a mapping")
    return _deep_copy(loaded)


def _deep_copy(value: Any) -> Any:
    if isinstance(value, Mapping):
        out = {}
        for k, v in value.items():
            if not isinstance(k, str):
                raise ConfigLoadError(f"configuration keys must be strings, got {k!r}")
            out[k] = _deep_copy(v)
        return out
    if isinstance(value, list):
        return [_deep_copy(v) for v in value]
    return value


def _env_world_size(world_size: int | None) -> int | None:
    if world_size is not None or "WORLD_SIZE" not in os.environ:
        return world_size
    try:
        return int(os.environ["WORLD_SIZE"])
    except ValueError as error:
        raise ConfigLoadError("WORLD_SIZE must be an integer") from error


def load_config(path: str | Path, *, overrides: Sequence[str] = (), world_size: int | None = None,
                emit_warnings: bool = True) -> TrainConfig:
    raw = _read_mapping(Path(path))
    for item in overrides:
        apply_override(raw, item)
    config = config_from_dict(raw)
    result = validate_config(config, world_size=_env_world_size(world_size))
    if emit_warnings:
        for message in result.warnings:
            warnings.warn(message, ConfigWarning, stacklevel=2)
    return config


def load_config_with_result(path: str | Path, *, overrides: Sequence[str] = (),
                            world_size: int | None = None
                            ) -> tuple[TrainConfig, ValidationResult]:
    config = load_config(path, overrides=overrides, world_size=world_size, emit_warnings=False)
    return config, validate_config(config, world_size=_env_world_size(world_size))
