"""Dataclass configs built from the composed YAML tree.

Every YAML node the trainers read is turned into a validated dataclass (the reference does
this with ``_target_`` + ``omega_conf_to_dataclass``; e.g. ``DiffusionAlgoConfig`` at
``verl_omni/trainer/config/algorithm.py:29``).  Unknown keys are kept in ``extra`` and
reported once, so configs written for the reference still load.
"""

from __future__ import annotations

import dataclasses
import logging
import typing
from typing import Any, Optional, get_args, get_origin

_log = logging.getLogger(__name__)


@dataclasses.dataclass
class BaseConfig:
    """Dataclass base with dict-style access and recursive construction from a mapping."""

    def get(self, key: str, default: Any = None) -> Any:
        return getattr(self, key, default)

    def __getitem__(self, key: str) -> Any:
        return getattr(self, key)

    def __contains__(self, key: str) -> bool:
        return hasattr(self, key)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    @classmethod
    def from_cfg(cls, cfg: Optional[dict], strict: bool = False):
        if cfg is None:
            return cls()
        if isinstance(cfg, cls):
            return cfg
        hints = typing.get_type_hints(cls)
        kwargs = {}
        unknown = []
        names = {f.name for f in dataclasses.fields(cls)}
        for k, v in dict(cfg).items():
            if k.startswith("_"):
                continue
            if k not in names:
                unknown.append(k)
                continue
            kwargs[k] = _coerce(hints.get(k), v)
        if unknown:
            if strict:
                raise KeyError(f"{cls.__name__}: unknown keys {unknown}")
            _log.debug("%s ignores unknown keys %s", cls.__name__, unknown)
        return cls(**kwargs)


def _coerce(tp: Any, value: Any) -> Any:
    if tp is None or value is None:
        return value
    origin = get_origin(tp)
    if origin is typing.Union or str(origin) == "types.UnionType":
        for arg in get_args(tp):
            if arg is type(None):
                continue
            try:
                return _coerce(arg, value)
            except (TypeError, ValueError):
                continue
        return value
    if isinstance(tp, type) and dataclasses.is_dataclass(tp) and issubclass(tp, BaseConfig) and isinstance(value, dict):
        return tp.from_cfg(value)
    if tp is float and isinstance(value, (int, str)) and not isinstance(value, bool):
        return float(value)
    if tp is int and isinstance(value, str) and value.lstrip("-").isdigit():
        return int(value)
    if origin in (list, tuple) and isinstance(value, (list, tuple)):
        return list(value)
    return value
