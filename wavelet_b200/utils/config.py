"""Command-line configuration loading.

Grammar (same as the reference's ``load_config``, utils/config.py:166-215):

    <cmd> [@ a.yaml] [@b.yaml] [--section.key VALUE] [--flag] [--no-flag] [--help]

* ``@ file`` / ``@file`` deep-merge YAML files left to right;
* ``--dotted.key VALUE`` sets a nested key; VALUE is parsed as JSON when it
  parses (numbers, lists, objects, true/false/null) and kept as a string
  otherwise; dashes in key parts become underscores;
* ``--flag`` with no value sets a boolean field true, ``--no-flag`` false;
* ``--help`` prints every flag of the schema with its type and default.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Literal, TypeVar, get_args, get_origin

import yaml
from pydantic import BaseModel

T = TypeVar("T", bound=BaseModel)


# ----------------------------------------------------------------------- YAML
class _StrictLoader(yaml.SafeLoader):
    """SafeLoader that rejects duplicate mapping keys (``<<`` merges allowed)."""


def _no_duplicates(loader: _StrictLoader, node: yaml.MappingNode, deep: bool = False):
    keys = []
    for k, _ in node.value:
        key = "<<" if k.tag == "tag:yaml.org,2002:merge" else loader.construct_object(k, deep=deep)
        if key in keys and key != "<<":
            raise yaml.constructor.ConstructorError(
                "while constructing a mapping", node.start_mark, f"found duplicate key {key!r}", k.start_mark
            )
        keys.append(key)
    return loader.construct_mapping(node, deep=deep)


_StrictLoader.add_constructor(yaml.resolver.BaseResolver.DEFAULT_MAPPING_TAG, _no_duplicates)


def load_yaml(path: Path | str) -> dict[str, Any]:
    with open(path, encoding="utf-8") as f:
        data = yaml.load(f, Loader=_StrictLoader)
    if data is None:
        return {}
    if not isinstance(data, dict):
        raise TypeError(f"Expected a mapping at the top of {path}")
    return data


def dump_yaml(path: Path | str, data: dict[str, Any]) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    with p.open("w", encoding="utf-8") as f:
        yaml.safe_dump(data, f, sort_keys=False)


def config_to_plain(cfg: BaseModel) -> dict[str, Any]:
    """JSON-safe dict of a config with secrets redacted."""
    return json.loads(cfg.model_dump_json())


# --------------------------------------------------------------------- merging
def merge(a: dict[str, Any], b: dict[str, Any]) -> dict[str, Any]:
    out = dict(a)
    for k, v in b.items():
        out[k] = merge(out[k], v) if isinstance(out.get(k), dict) and isinstance(v, dict) else v
    return out


def _assign(tree: dict[str, Any], dotted: str, value: Any) -> None:
    *parents, leaf = dotted.split(".")
    node = tree
    for p in parents:
        nxt = node.setdefault(p, {})
        if nxt is None:
            nxt = node[p] = {}
        if not isinstance(nxt, dict):
            raise TypeError(f"Cannot override nested key '{dotted}': '{p}' is not a section.")
        node = nxt
    node[leaf] = value


def _coerce(text: str) -> Any:
    try:
        return json.loads(text)
    except json.JSONDecodeError:
        return text


# ------------------------------------------------------------------ schema walk
def _submodels(ann: Any) -> list[type[BaseModel]]:
    if isinstance(ann, type) and issubclass(ann, BaseModel):
        return [ann]
    found: list[type[BaseModel]] = []
    for a in get_args(ann):
        for m in _submodels(a):
            if m not in found:
                found.append(m)
    return found


def _has_bool(ann: Any) -> bool:
    return ann is bool or any(_has_bool(a) for a in get_args(ann))


def _is_boolean_key(schema: type[BaseModel], dotted: str) -> bool:
    models = [schema]
    anns: list[Any] = []
    parts = dotted.split(".")
    for i, part in enumerate(parts):
        anns = [m.model_fields[part].annotation for m in models if part in m.model_fields]
        if i < len(parts) - 1:
            models = [sm for a in anns for sm in _submodels(a)]
    return bool(anns) and all(_has_bool(a) for a in anns)


def _label(ann: Any) -> str:
    names = {bool: "BOOL", str: "STR", int: "INT", float: "FLOAT", Path: "PATH"}
    if ann in names:
        return names[ann]
    if get_origin(ann) is Literal:
        return "{" + ",".join(map(str, get_args(ann))) + "}"
    origin = get_origin(ann)
    if origin is not None:
        return getattr(origin, "__name__", str(origin)).upper()
    return getattr(ann, "__name__", "VALUE").upper()


def help_text(schema: type[BaseModel]) -> str:
    rows: dict[str, tuple[str, str]] = {}

    def walk(model: type[BaseModel], prefix: str, seen: tuple):
        for name, f in model.model_fields.items():
            key = f"{prefix}.{name}" if prefix else name
            subs = [m for m in _submodels(f.annotation) if m not in seen]
            if subs:
                for m in subs:
                    walk(m, key, seen + (model,))
                continue
            flag = "--" + key.replace("_", "-")
            lab = "BOOL (also --no-...)" if _has_bool(f.annotation) else _label(f.annotation)
            desc = f.description or ""
            if not f.is_required() and isinstance(f.default, (str, int, float, bool, type(None), Path)):
                desc = f"{desc} [default: {f.default}]".strip()
            rows.setdefault(flag, (lab, desc))

    walk(schema, "", ())
    w = max((len(k) for k in rows), default=0)
    out = [f"{schema.__name__} configuration", "Usage: [@ CONFIG ...] [--field VALUE] [--flag | --no-flag]", "", "Options:"]
    out += [f"  {k:<{w}}  {lab}" + (f"  {d}" if d else "") for k, (lab, d) in rows.items()]
    return "\n".join(out)


# ----------------------------------------------------------------------- entry
def parse_argv(schema: type[BaseModel], argv: list[str]) -> dict[str, Any]:
    data: dict[str, Any] = {}
    rest: list[str] = []
    it = iter(range(len(argv)))
    i = 0
    while i < len(argv):
        tok = argv[i]
        if tok == "@":
            if i + 1 >= len(argv):
                raise SystemExit("Expected a path after '@'.")
            data = merge(data, load_yaml(argv[i + 1]))
            i += 2
        elif tok.startswith("@") and len(tok) > 1:
            data = merge(data, load_yaml(tok[1:]))
            i += 1
        else:
            rest.append(tok)
            i += 1
    del it
    j = 0
    while j < len(rest):
        tok = rest[j]
        if not tok.startswith("--"):
            raise SystemExit(f"Invalid override '{tok}'. Expected --section.key.")
        name = tok[2:]
        neg = name.startswith("no-")
        if neg:
            name = name[3:]
        key = ".".join(p.replace("-", "_") for p in name.split("."))
        if not key:
            raise SystemExit("Configuration override names cannot be empty.")
        nxt_is_flag = j + 1 >= len(rest) or rest[j + 1].startswith("--")
        if neg:
            val: Any = False
            j += 1
        elif nxt_is_flag and _is_boolean_key(schema, key):
            val = True
            j += 1
        else:
            if j + 1 >= len(rest):
                raise SystemExit(f"Expected a value after '{tok}'.")
            val = _coerce(rest[j + 1])
            j += 2
        _assign(data, key, val)
    return data


def load_config(schema: type[T], argv: list[str]) -> T:
    if "--help" in argv or "-h" in argv:
        print(help_text(schema))
        raise SystemExit(0)
    return schema.model_validate(parse_argv(schema, argv))
