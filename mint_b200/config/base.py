"""Dataclass configuration tree loaded from TOML.

Same schema semantics as the reference (mint/config/base.py:8-47): every config is a
dataclass; nested dataclass fields (including ``X | None`` unions) are built
recursively from TOML tables; unknown keys raise ``TypeError`` from the dataclass
constructor.
"""

from __future__ import annotations

import tomllib
import types
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Any, Self, Union, get_args, get_origin, get_type_hints


def _config_type_of(field_type: Any) -> Any:  # noqa: ANN401
    """Return the Config subclass inside ``field_type`` (plain or a union), else ``field_type``."""
    if get_origin(field_type) in (Union, types.UnionType):
        for arg in get_args(field_type):
            if isinstance(arg, type) and issubclass(arg, Config):
                return arg
    return field_type


@dataclass
class Config:
    @classmethod
    def _field_types(cls) -> dict[str, Any]:
        try:
            hints = get_type_hints(cls)
        except Exception:  # noqa: BLE001 - forward refs that cannot resolve fall back to raw annotations
            hints = {}
        return {f.name: hints.get(f.name, f.type) for f in fields(cls)}

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> Self:
        types_by_name = cls._field_types()
        kwargs: dict[str, Any] = {}
        for key, value in data.items():
            target = _config_type_of(types_by_name.get(key))
            if isinstance(value, dict) and isinstance(target, type) and issubclass(target, Config):
                kwargs[key] = target.from_dict(value)
            else:
                kwargs[key] = value
        return cls(**kwargs)

    @classmethod
    def from_toml(cls, toml_path: str) -> Self:
        path = Path(toml_path)
        if not path.exists():
            raise FileNotFoundError(f"Config file not found: {toml_path}")
        with path.open("rb") as fh:
            return cls.from_dict(tomllib.load(fh))
