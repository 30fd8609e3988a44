"""Typed run configuration: YAML files mapped onto trees of dataclasses.

The file format is the one the upstream project uses (reference:
``src/myk_llm/configuration.py:1-146``) so that every YAML config written for it loads
here unchanged:

* ``base:`` at the top of a file names one file or a list of files to inherit from,
  resolved against the including file's directory.  Mappings merge key by key,
  recursively; scalars and lists from the child replace the parent's.
* Overrides on the command line look like ``a.b.c=value``; the value is parsed as YAML
  (``3e-4``, ``true``, ``[2, 3]``, ``null``).
* A key that the dataclass does not declare is an error, and values are checked
  against the field annotations (``Union``/``Optional``, ``Literal``, ``list``,
  ``tuple``, ``dict``, nested dataclasses).  YAML reads ``3e-4`` as a string; a string
  is accepted for a ``float`` field when it parses as one.

The implementation is a small recursive validator: ``_check`` walks the annotation and
the value together and returns the converted value or raises with the dotted path.
"""

from __future__ import annotations

import dataclasses
import types
import typing
from pathlib import Path
from typing import Any, TypeVar

import yaml

T = TypeVar("T")

__all__ = [
    "apply_overrides",
    "dump_yaml",
    "from_dict",
    "load_config",
    "load_yaml_tree",
    "merge_trees",
    "to_dict",
]


def merge_trees(parent: dict[str, Any], child: dict[str, Any]) -> dict[str, Any]:
    """Recursive mapping merge; the child wins everywhere except inside mappings."""
    out = dict(parent)
    for key, value in child.items():
        prev = out.get(key)
        out[key] = merge_trees(prev, value) if isinstance(prev, dict) and isinstance(value, dict) else value
    return out


def load_yaml_tree(path: str | Path) -> dict[str, Any]:
    """Read a YAML file and fold in its ``base:`` chain (depth first, in list order)."""
    path = Path(path)
    tree = yaml.safe_load(path.read_text(encoding="utf-8")) or {}
    if not isinstance(tree, dict):
        raise ValueError(f"{path}: a config file must hold a mapping at the top level")
    bases = tree.pop("base", None)
    if bases is None:
        return tree
    if isinstance(bases, (str, Path)):
        bases = [bases]
    inherited: dict[str, Any] = {}
    for base in bases:
        inherited = merge_trees(inherited, load_yaml_tree(path.parent / base))
    return merge_trees(inherited, tree)


def apply_overrides(tree: dict[str, Any], overrides: list[str] | None) -> dict[str, Any]:
    """Return a copy of ``tree`` with each ``dotted.key=yaml`` override applied."""
    out = dict(tree)
    for item in overrides or []:
        key, sep, raw = item.partition("=")
        if not sep:
            raise ValueError(f"override {item!r} must look like key.path=value")
        parts = key.strip().split(".")
        node = out
        for part in parts[:-1]:
            child = node.get(part)
            node[part] = dict(child) if isinstance(child, dict) else {}
            node = node[part]
        node[parts[-1]] = yaml.safe_load(raw)
    return out


def _check(value: Any, ann: Any, path: str) -> Any:
    if ann is Any:
        return value
    origin, args = typing.get_origin(ann), typing.get_args(ann)
    if origin is typing.Union or origin is types.UnionType:
        if value is None and type(None) in args:
            return None
        problems = []
        for option in args:
            if option is type(None):
                continue
            try:
                return _check(value, option, path)
            except (TypeError, ValueError) as err:
                problems.append(str(err))
        raise TypeError(f"{path}: {value!r} fits none of {ann} ({'; '.join(problems)})")
    if origin is typing.Literal:
        if value not in args:
            raise ValueError(f"{path}: {value!r} is not one of {args}")
        return value
    if dataclasses.is_dataclass(ann) and isinstance(ann, type):
        if isinstance(value, ann):
            return value
        if not isinstance(value, dict):
            raise TypeError(f"{path}: expected a mapping for {ann.__name__}, got {value!r}")
        return from_dict(ann, value, path)
    if origin in (list, tuple):
        if not isinstance(value, (list, tuple)):
            raise TypeError(f"{path}: expected a list, got {value!r}")
        item_ann = args[0] if args else Any
        items = [_check(v, item_ann, f"{path}[{i}]") for i, v in enumerate(value)]
        return items if origin is list else tuple(items)
    if origin is dict:
        if not isinstance(value, dict):
            raise TypeError(f"{path}: expected a mapping, got {value!r}")
        val_ann = args[1] if len(args) == 2 else Any
        return {k: _check(v, val_ann, f"{path}.{k}") for k, v in value.items()}
    if ann is float:
        if isinstance(value, bool):
            raise TypeError(f"{path}: expected float, got {value!r}")
        if isinstance(value, (int, float)):
            return float(value)
        if isinstance(value, str):
            return float(value)
        raise TypeError(f"{path}: expected float, got {value!r}")
    if ann is int:
        if isinstance(value, bool) or not isinstance(value, int):
            raise TypeError(f"{path}: expected int, got {value!r}")
        return value
    if ann in (str, bool):
        if not isinstance(value, ann):
            raise TypeError(f"{path}: expected {ann.__name__}, got {value!r}")
        return value
    return value


def from_dict(cls: type[T], data: dict[str, Any], where: str = "") -> T:
    """Build dataclass ``cls`` from a plain mapping, validating every field."""
    hints = typing.get_type_hints(cls)
    names = {f.name for f in dataclasses.fields(cls)}  # type: ignore[arg-type]
    extra = sorted(set(data) - names)
    if extra:
        raise KeyError(f"{where or cls.__name__}: unknown key(s) {extra}; known: {sorted(names)}")
    kwargs = {k: _check(v, hints[k], f"{where}.{k}" if where else k) for k, v in data.items()}
    return cls(**kwargs)


def to_dict(obj: Any) -> Any:
    """Plain-Python (YAML-safe) view of a dataclass tree."""
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        return {f.name: to_dict(getattr(obj, f.name)) for f in dataclasses.fields(obj)}
    if isinstance(obj, (list, tuple)):
        return [to_dict(v) for v in obj]
    if isinstance(obj, dict):
        return {k: to_dict(v) for k, v in obj.items()}
    return obj


def load_config(cls: type[T], path: str | Path | None, overrides: list[str] | None = None) -> T:
    tree = load_yaml_tree(path) if path else {}
    return from_dict(cls, apply_overrides(tree, overrides))


def dump_yaml(config: Any) -> str:
    return yaml.safe_dump(to_dict(config), sort_keys=False, allow_unicode=True)
