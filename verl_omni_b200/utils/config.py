"""Hierarchical YAML configuration with defaults composition, interpolation and CLI overrides.

The reference drives everything through Hydra + OmegaConf
(``verl_omni/trainer/config/diffusion_trainer.yaml:8-37``): a defaults list composes
per-component YAML files at package paths (``diffusion/actor@actor_rollout_ref.actor``),
values cross-link with ``${oc.select:path,default}`` and users override any key on the
command line (``actor_rollout_ref.rollout.n=16``, ``+new.key=1``).  Neither Hydra nor
OmegaConf is a dependency here, so this module implements the subset of that behaviour the
trainers use, keeping the same key paths and override syntax:

* ``defaults:`` entries ``group@target.path: name`` / ``group: name`` / ``_self_``;
  ``${group}`` inside a default name resolves to an earlier selection.
* interpolation: ``${a.b.c}`` (absolute), ``${.x}`` (sibling), ``${oc.select:a.b,dflt}``,
  ``${oc.env:VAR,dflt}``.  Whole-string interpolations keep the target's type.
* CLI overrides ``a.b=v`` (key must exist unless ``+`` prefixed), ``++a.b=v`` (force),
  ``~a.b`` (delete); values parse as YAML scalars/lists.
"""

from __future__ import annotations

import copy
import os
import re
from pathlib import Path
from typing import Optional, Any, Iterable

import yaml

CONFIG_ROOT = Path(__file__).resolve().parent.parent / "trainer" / "config"

_MISSING = "???"


class Cfg(dict):
    """A dict with attribute access, dotted ``get`` and ``select`` helpers."""

    def __getattr__(self, item):
        try:
            return self[item]
        except KeyError as e:  # attribute protocol needs AttributeError
            raise AttributeError(item) from e

    def __setattr__(self, key, value):
        self[key] = value

    def __delattr__(self, item):
        del self[item]

    def __deepcopy__(self, memo):
        return Cfg({k: copy.deepcopy(v, memo) for k, v in self.items()})

    def select(self, path: str, default: Any = None) -> Any:
        node: Any = self
        for part in path.split("."):
            if isinstance(node, dict) and part in node:
                node = node[part]
            else:
                return default
        return node

    def to_dict(self) -> dict:
        return to_plain(self)


def to_cfg(obj: Any) -> Any:
    if isinstance(obj, Cfg):
        return Cfg({k: to_cfg(v) for k, v in obj.items()})
    if isinstance(obj, dict):
        return Cfg({k: to_cfg(v) for k, v in obj.items()})
    if isinstance(obj, list):
        return [to_cfg(v) for v in obj]
    return obj


def to_plain(obj: Any) -> Any:
    if isinstance(obj, dict):
        return {k: to_plain(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [to_plain(v) for v in obj]
    return obj


def _deep_merge(base: dict, override: dict) -> dict:
    for k, v in override.items():
        if k == "defaults":
            continue
        if isinstance(v, dict) and isinstance(base.get(k), dict):
            _deep_merge(base[k], v)
        else:
            base[k] = copy.deepcopy(v)
    return base


def _set_path(root: dict, path: str, value: Any, create: bool = True) -> None:
    parts = path.split(".")
    node = root
    for p in parts[:-1]:
        if p not in node or not isinstance(node[p], dict):
            if not create:
                raise KeyError(f"config path {path!r} does not exist")
            node[p] = Cfg()
        node = node[p]
    if not create and parts[-1] not in node:
        raise KeyError(f"config key {path!r} does not exist (prefix it with '+' to add it)")
    node[parts[-1]] = value


def _get_path(root: dict, path: str) -> Any:
    node: Any = root
    for p in path.split("."):
        if not isinstance(node, dict) or p not in node:
            raise KeyError(path)
        node = node[p]
    return node


def _del_path(root: dict, path: str) -> None:
    parts = path.split(".")
    node = _get_path(root, ".".join(parts[:-1])) if len(parts) > 1 else root
    node.pop(parts[-1], None)


def _load_yaml(path: Path) -> dict:
    with open(path) as f:
        data = yaml.safe_load(f) or {}
    return data


def compose(name: str, root: Path = CONFIG_ROOT, choices: Optional[dict] = None) -> Cfg:
    """Compose the config ``<root>/<name>.yaml`` with its defaults list (recursively); ``choices`` replaces
    the option a defaults entry selects for a group (Hydra's ``group=option`` overrides)."""
    return to_cfg(_compose_file(root / f"{name}.yaml", root, selections={"__choices__": dict(choices or {})}))


def _compose_file(path: Path, root: Path, selections: dict) -> dict:
    raw = _load_yaml(path)
    defaults = raw.get("defaults", [])
    result: dict = {}
    self_applied = False
    for entry in defaults:
        if entry == "_self_":
            _deep_merge(result, raw)
            self_applied = True
            continue
        if isinstance(entry, str):
            sub = _compose_file(path.parent / f"{entry}.yaml", root, selections)
            _deep_merge(result, sub)
            continue
        ((key, val),) = entry.items()
        if val is None:
            continue
        val = re.sub(r"\$\{([^}]+)\}", lambda m: str(selections.get(m.group(1), m.group(0))), str(val))
        group, _, target = key.partition("@")
        val = selections.get("__choices__", {}).get(group, val)
        selections[group] = val
        group_dir = root / group
        sub = _compose_file(group_dir / f"{val}.yaml", root, selections)
        if target:
            holder: dict = {}
            node = holder
            parts = target.split(".")
            for p in parts[:-1]:
                node = node.setdefault(p, {})
            node[parts[-1]] = sub
            _deep_merge(result, holder)
        else:
            # a plain group selection (no @package) merges at the root only when the
            # selected file is a top-level fragment; a bare selection like
            # ``diffusion/model_engine: dp_diffusion`` only records the choice.
            if sub:
                _deep_merge(result, sub)
    if not self_applied:
        _deep_merge(result, raw)
    return result


def parse_value(text: str) -> Any:
    try:
        return yaml.safe_load(text)
    except yaml.YAMLError:
        return text


def apply_overrides(cfg: Cfg, overrides: Iterable[str]) -> Cfg:
    for ov in overrides:
        ov = ov.strip()
        if not ov:
            continue
        if ov.startswith("~"):
            _del_path(cfg, ov[1:].split("=")[0])
            continue
        force = ov.startswith("++")
        add = ov.startswith("+") and not force
        key, sep, val = ov.lstrip("+").partition("=")
        if not sep:
            raise ValueError(f"override {ov!r} must be key=value")
        _set_path(cfg, key, to_cfg(parse_value(val)), create=(add or force))
    return cfg


_INTERP = re.compile(r"\$\{([^${}]+)\}")


def _resolve_expr(expr: str, root: dict, parent_path: list[str]) -> Any:
    expr = expr.strip()
    if expr.startswith("oc.select:"):
        body = expr[len("oc.select:"):]
        path, _, default = body.partition(",")
        try:
            return _lookup(path.strip(), root, parent_path)
        except KeyError:
            return parse_value(default.strip()) if default.strip() else None
    if expr.startswith("oc.env:"):
        body = expr[len("oc.env:"):]
        var, _, default = body.partition(",")
        v = os.environ.get(var.strip())
        return parse_value(v) if v is not None else parse_value(default.strip())
    return _lookup(expr, root, parent_path)


def _lookup(path: str, root: dict, parent_path: list[str]) -> Any:
    if path.startswith("."):
        # relative: count leading dots (one dot = sibling)
        n = len(path) - len(path.lstrip("."))
        base = parent_path[: len(parent_path) - (n - 1)] if n > 1 else parent_path
        path = ".".join(base + [path.lstrip(".")])
    value = _get_path(root, path)
    if value == _MISSING:
        raise KeyError(path)
    return value


def resolve(cfg: Cfg, max_passes: int = 16) -> Cfg:
    """Resolve every interpolation in place (iterates until a fixed point)."""

    def walk(node: Any, path: list[str]) -> tuple[Any, bool]:
        changed = False
        if isinstance(node, dict):
            for k in list(node.keys()):
                node[k], c = walk(node[k], path + [str(k)])
                changed |= c
            return node, changed
        if isinstance(node, list):
            for i, v in enumerate(node):
                node[i], c = walk(v, path)
                changed |= c
            return node, changed
        if isinstance(node, str) and "${" in node:
            parent = path[:-1]
            m = _INTERP.fullmatch(node.strip())
            if m:
                try:
                    val = _resolve_expr(m.group(1), cfg, parent)
                except KeyError:
                    return node, False
                if isinstance(val, str) and "${" in val:
                    return val, True
                return copy.deepcopy(to_cfg(val)), True

            def sub(mm):
                try:
                    return str(_resolve_expr(mm.group(1), cfg, parent))
                except KeyError:
                    return mm.group(0)

            new = _INTERP.sub(sub, node)
            return new, new != node
        return node, False

    for _ in range(max_passes):
        _, changed = walk(cfg, [])
        if not changed:
            break
    return cfg


def load_config(name: str = "diffusion_trainer", overrides: Iterable[str] = (), root: Path = CONFIG_ROOT) -> Cfg:
    """Compose + override + resolve: the equivalent of ``@hydra.main`` followed by ``OmegaConf.resolve``.

    An override whose key names a config group directory (``diffusion/model_engine=veomni_diffusion``)
    selects that group's option in the defaults lists; every other override sets a value."""
    choices, rest = {}, []
    for ov in overrides:
        key, sep, val = ov.strip().partition("=")
        if sep and "/" in key and "." not in key and (root / key).is_dir():
            choices[key] = val
        else:
            rest.append(ov)
    cfg = compose(name, root, choices)
    apply_overrides(cfg, rest)
    return resolve(cfg)
