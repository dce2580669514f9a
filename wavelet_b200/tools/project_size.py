"""``python -m wavelet_b200.tools.project_size``: files, lines and a rough
Python complexity count of this project, as one JSON snapshot (optionally
appended to a JSONL history with ``--write``) (reference
scripts/project_size.py).

Files: ``git ls-files`` when the root is a git work tree, else a walk that
skips caches, virtualenvs and outputs; counted suffixes are source, config and
documentation types (``.py .cu .cuh .cpp .h .md .yaml .yml .toml .json .html
.js .css``).  Per file: total, source, blank and comment lines (``#`` for
Python/YAML/TOML, ``//`` for C++/CUDA); for Python also functions, classes
and complexity points (one per branch, loop, handler, boolean operator,
comprehension, with, assert and match).  Files are grouped by category from
their path (package subpackage, tests, examples, profiles, ...).
"""

from __future__ import annotations

import argparse
import ast
import json
import subprocess
from collections import Counter
from datetime import datetime, timezone
from pathlib import Path

SUFFIXES = {".py", ".cu", ".cuh", ".cpp", ".h", ".md", ".yaml", ".yml", ".toml", ".json", ".html", ".js", ".css"}
SKIP = {".git", "__pycache__", ".pytest_cache", ".venv", "outputs", "_build", "_work", "baseline"}
COMMENT = {".py": "#", ".yaml": "#", ".yml": "#", ".toml": "#", ".cu": "//", ".cuh": "//", ".cpp": "//", ".h": "//",
           ".js": "//", ".css": "/*"}
BRANCHES = (ast.If, ast.For, ast.While, ast.Try, ast.ExceptHandler, ast.With, ast.BoolOp, ast.IfExp, ast.Assert,
            ast.comprehension, ast.Match)
CORE = {"csrc", "models", "ops", "parallel", "trainer", "inference", "orchestrator", "data", "configs", "utils",
        "transport", "entrypoints", "environments", "dashboard", "deployment", "tools", "package"}


def project_files(root: Path) -> list[Path]:
    try:
        out = subprocess.run(["git", "ls-files"], cwd=root, capture_output=True, text=True, check=True).stdout
        paths = [root / p for p in out.splitlines()]
    except (OSError, subprocess.CalledProcessError):
        paths = [p for p in root.rglob("*") if p.is_file()]
    return sorted(p for p in paths if p.is_file() and p.suffix in SUFFIXES
                  and not any(part in SKIP for part in p.relative_to(root).parts))


def category(rel: str) -> str:
    parts = rel.split("/")
    if parts[0] == "wavelet_b200":
        return parts[1] if len(parts) > 2 else "package"
    return {"tests": "tests", "examples": "examples", "profiles": "profiles"}.get(parts[0], "other")


def measure(root: Path, path: Path) -> dict:
    rel = path.relative_to(root).as_posix()
    text = path.read_text(errors="replace")
    lines = text.splitlines()
    blank = sum(1 for ln in lines if not ln.strip())
    mark = COMMENT.get(path.suffix)
    comment = sum(1 for ln in lines if mark and ln.strip().startswith(mark))
    m = {"path": rel, "suffix": path.suffix, "category": category(rel), "lines": len(lines), "blank_lines": blank,
         "comment_lines": comment, "source_lines": len(lines) - blank - comment, "python_functions": 0,
         "python_classes": 0, "python_complexity_points": 0}
    if path.suffix == ".py":
        try:
            tree = ast.parse(text)
        except SyntaxError:
            return m
        for node in ast.walk(tree):
            if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef)):
                m["python_functions"] += 1
            elif isinstance(node, ast.ClassDef):
                m["python_classes"] += 1
            elif isinstance(node, BRANCHES):
                m["python_complexity_points"] += 1
    return m


def summarize(files: list[dict], timestamp: str | None = None, top: int = 12) -> dict:
    fields = ("lines", "source_lines", "python_functions", "python_classes", "python_complexity_points")
    totals = {f: sum(x[f] for x in files) for f in fields}
    by_cat: dict[str, dict] = {}
    for x in files:
        c = by_cat.setdefault(x["category"], {"files": 0, **{f: 0 for f in fields}})
        c["files"] += 1
        for f in fields:
            c[f] += x[f]
    core = sum(v["source_lines"] for k, v in by_cat.items() if k in CORE)
    return {"timestamp": timestamp or datetime.now(timezone.utc).isoformat(timespec="seconds"),
            "files": len(files), **totals, "core_source_lines": core,
            "by_suffix": dict(sorted(Counter(x["suffix"] for x in files).items())),
            "by_category": dict(sorted(by_cat.items())),
            "largest": [{"path": x["path"], "lines": x["lines"]}
                        for x in sorted(files, key=lambda x: -x["lines"])[:top]]}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Count project files, lines and rough Python complexity.")
    ap.add_argument("--root", type=Path, default=Path.cwd())
    ap.add_argument("--write", type=Path, help="append the snapshot to this JSONL file")
    ap.add_argument("--timestamp")
    ap.add_argument("--top", type=int, default=12)
    a = ap.parse_args(argv)
    root = a.root.resolve()
    snap = summarize([measure(root, p) for p in project_files(root)], a.timestamp, a.top)
    line = json.dumps(snap, sort_keys=True)
    print(line)
    if a.write is not None:
        out = a.write if a.write.is_absolute() else root / a.write
        out.parent.mkdir(parents=True, exist_ok=True)
        with out.open("a") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
