"""YAML configuration loading for rl_b200.

Implements the configuration behaviour of the reference's OmegaConf/Hydra layer
(reference: ``nemo_rl/utils/config.py:53`` defaults inheritance, ``:102``
``load_config``, ``:174`` ``parse_hydra_overrides``, ``:230`` the ``${mul:a,b}``
resolver) without depending on OmegaConf, which is not part of this stack.

Supported features
------------------
* ``defaults: "base.yaml"`` or ``defaults: [a.yaml, b.yaml]`` - files are loaded
  relative to the including file and deep-merged, later entries and the child
  file winning.
* Interpolation ``${a.b.c}`` (absolute path), ``${.x}`` / ``${..x}`` (relative to
  the node holding the value) and resolvers ``${mul:x,y}``, ``${div:x,y}``,
  ``${add:x,y}``, ``${max:x,y}``, ``${min:x,y}``.  A value that is exactly one
  interpolation keeps the referenced type; interpolations embedded in a longer
  string are substituted textually.
* Command-line overrides ``a.b=1`` (key must exist), ``+a.b=1`` (new key),
  ``++a.b=1`` (set whether or not it exists) and ``~a.b`` (delete).
"""

from __future__ import annotations

import copy
import os
import re
from typing import Any, Iterable, Optional

import yaml

__all__ = [
    "load_config",
    "load_config_with_inheritance",
    "merge_configs",
    "resolve_interpolations",
    "apply_overrides",
    "parse_overrides",
    "get_by_path",
    "set_by_path",
]

_INTERP = re.compile(r"\$\{([^${}]+)\}")


def merge_configs(base: dict, override: dict) -> dict:
    """Deep-merge ``override`` into a copy of ``base`` (dicts merge, everything else replaces)."""
    out = copy.deepcopy(base)
    for key, val in override.items():
        if isinstance(val, dict) and isinstance(out.get(key), dict):
            out[key] = merge_configs(out[key], val)
        else:
            out[key] = copy.deepcopy(val)
    return out


def load_config_with_inheritance(path: str, _seen: Optional[set] = None) -> dict:
    """Load ``path`` and recursively merge the files named in its ``defaults`` key."""
    path = os.path.abspath(path)
    seen = set() if _seen is None else _seen
    if path in seen:
        raise ValueError(f"cyclic 'defaults' inheritance through {path}")
    seen = seen | {path}
    with open(path) as f:
        cfg = yaml.safe_load(f) or {}
    if not isinstance(cfg, dict):
        raise ValueError(f"top level of {path} must be a mapping")
    defaults = cfg.pop("defaults", None)
    if defaults is None:
        return cfg
    if isinstance(defaults, str):
        defaults = [defaults]
    merged: dict = {}
    here = os.path.dirname(path)
    for parent in defaults:
        parent_path = parent if os.path.isabs(parent) else os.path.join(here, parent)
        merged = merge_configs(merged, load_config_with_inheritance(parent_path, seen))
    return merge_configs(merged, cfg)


def get_by_path(cfg: Any, dotted: str) -> Any:
    node = cfg
    for part in dotted.split("."):
        if isinstance(node, dict):
            if part not in node:
                raise KeyError(dotted)
            node = node[part]
        elif isinstance(node, list):
            node = node[int(part)]
        else:
            raise KeyError(dotted)
    return node


def set_by_path(cfg: dict, dotted: str, value: Any, create: bool = True) -> None:
    parts = dotted.split(".")
    node = cfg
    for part in parts[:-1]:
        if isinstance(node, list):
            node = node[int(part)]
            continue
        if part not in node or node[part] is None:
            if not create:
                raise KeyError(dotted)
            node[part] = {}
        node = node[part]
    if isinstance(node, list):
        node[int(parts[-1])] = value
    else:
        node[parts[-1]] = value


def _num(x: Any) -> Any:
    if isinstance(x, str):
        try:
            return int(x)
        except ValueError:
            return float(x)
    return x


_RESOLVERS = {
    "mul": lambda a, b: _num(a) * _num(b),
    "div": lambda a, b: _num(a) / _num(b),
    "floordiv": lambda a, b: _num(a) // _num(b),
    "add": lambda a, b: _num(a) + _num(b),
    "max": lambda a, b: max(_num(a), _num(b)),
    "min": lambda a, b: min(_num(a), _num(b)),
}


def _split_args(s: str) -> list[str]:
    """Split resolver arguments on top-level commas (``${mul:${a},2}`` already expanded)."""
    return [p.strip() for p in s.split(",")]


def resolve_interpolations(cfg: dict, max_passes: int = 32) -> dict:
    """Return a copy of ``cfg`` with every ``${...}`` expression resolved."""
    root = copy.deepcopy(cfg)

    def lookup(expr: str, where: list[str]) -> Any:
        expr = expr.strip()
        if ":" in expr and not expr.startswith("."):
            name, args = expr.split(":", 1)
            if name not in _RESOLVERS:
                raise KeyError(f"unknown resolver '{name}' in ${{{expr}}}")
            return _RESOLVERS[name](*_split_args(args))
        if expr.startswith("."):
            ups = len(expr) - len(expr.lstrip("."))
            rest = expr[ups:]
            base = where[: max(0, len(where) - ups)]
            dotted = ".".join(base + ([rest] if rest else []))
        else:
            dotted = expr
        return get_by_path(root, dotted)

    def resolve_value(val: Any, where: list[str]) -> tuple[Any, bool]:
        if not isinstance(val, str) or "${" not in val:
            return val, False
        m = _INTERP.fullmatch(val.strip())
        if m is not None and "${" not in m.group(1):
            got = lookup(m.group(1), where)
            if isinstance(got, str) and "${" in got:
                return val, False  # target not resolved yet
            return copy.deepcopy(got), True

        changed = False

        def sub(mm: re.Match) -> str:
            nonlocal changed
            got = lookup(mm.group(1), where)
            if isinstance(got, str) and "${" in got:
                return mm.group(0)
            changed = True
            return str(got)

        new = _INTERP.sub(sub, val)
        if changed and "${" not in new:
            try:
                parsed = yaml.safe_load(new)
                if isinstance(parsed, (int, float, bool)):
                    return parsed, True
            except yaml.YAMLError:
                pass
        return new, changed

    def walk(node: Any, where: list[str]) -> bool:
        changed = False
        if isinstance(node, dict):
            for k in list(node.keys()):
                v = node[k]
                if isinstance(v, (dict, list)):
                    changed |= walk(v, where + [str(k)])
                else:
                    nv, c = resolve_value(v, where + [str(k)])
                    if c:
                        node[k] = nv
                        changed = True
        elif isinstance(node, list):
            for i, v in enumerate(node):
                if isinstance(v, (dict, list)):
                    changed |= walk(v, where + [str(i)])
                else:
                    nv, c = resolve_value(v, where + [str(i)])
                    if c:
                        node[i] = nv
                        changed = True
        return changed

    for _ in range(max_passes):
        if not walk(root, []):
            break

    def leftover(node: Any) -> Optional[str]:
        if isinstance(node, dict):
            for v in node.values():
                r = leftover(v)
                if r:
                    return r
        elif isinstance(node, list):
            for v in node:
                r = leftover(v)
                if r:
                    return r
        elif isinstance(node, str) and _INTERP.search(node):
            return node
        return None

    bad = leftover(root)
    if bad is not None:
        raise ValueError(f"could not resolve interpolation {bad!r} (cycle or missing key)")
    return root


def parse_overrides(overrides: Iterable[str]) -> list[tuple[str, str, Any]]:
    """Parse Hydra-style overrides into ``(op, dotted_key, value)`` triples.

    ``op`` is one of ``set`` (key must exist), ``add`` (``+key``), ``force``
    (``++key``) or ``del`` (``~key``).
    """
    parsed = []
    for item in overrides:
        item = item.strip()
        if not item:
            continue
        if item.startswith("~"):
            parsed.append(("del", item[1:].split("=", 1)[0], None))
            continue
        if "=" not in item:
            raise ValueError(f"override '{item}' is not of the form key=value")
        key, raw = item.split("=", 1)
        op = "set"
        if key.startswith("++"):
            op, key = "force", key[2:]
        elif key.startswith("+"):
            op, key = "add", key[1:]
        value = yaml.safe_load(raw) if raw != "" else ""
        parsed.append((op, key, value))
    return parsed


def apply_overrides(cfg: dict, overrides: Iterable[str]) -> dict:
    out = copy.deepcopy(cfg)
    for op, key, value in parse_overrides(overrides):
        exists = True
        try:
            get_by_path(out, key)
        except (KeyError, IndexError, ValueError):
            exists = False
        if op == "del":
            if not exists:
                raise KeyError(f"cannot delete missing key '{key}'")
            parent, _, leaf = key.rpartition(".")
            node = get_by_path(out, parent) if parent else out
            del node[leaf]
        elif op == "set":
            if not exists:
                raise KeyError(
                    f"override key '{key}' is not in the config; use '+{key}=...' to add it"
                )
            set_by_path(out, key, value, create=False)
        elif op == "add":
            if exists:
                raise KeyError(f"key '{key}' already exists; use '++{key}=...' to replace it")
            set_by_path(out, key, value, create=True)
        else:
            set_by_path(out, key, value, create=True)
    return out


def load_config(path: str, overrides: Optional[Iterable[str]] = None, resolve: bool = True) -> dict:
    """Load a YAML config with ``defaults`` inheritance, CLI overrides and interpolation."""
    cfg = load_config_with_inheritance(path)
    if overrides:
        cfg = apply_overrides(cfg, overrides)
    return resolve_interpolations(cfg) if resolve else cfg
