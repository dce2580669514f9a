"""``wavelet dashboard``: serve the read-only dashboard over run directories
(reference entrypoints/dashboard.py:20-53)."""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

from ..dashboard.server import RunRegistry, build_app, default_static_dir


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="wavelet dashboard",
                                description="Serve a read-only dashboard over one or more run directories.")
    p.add_argument("runs", nargs="*", type=Path, help="run output directories to serve explicitly")
    p.add_argument("--runs-root", action="append", default=[], type=Path,
                   help="directory whose immediate children are run directories (repeatable)")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8766)
    p.add_argument("--static-dir", type=Path, default=default_static_dir())
    p.add_argument("--log-level", default="warning")
    return p


def main(argv: list[str] | None = None) -> int:
    a = build_parser().parse_args(sys.argv[1:] if argv is None else argv)
    if not a.runs and not a.runs_root:
        a.runs_root = [Path("outputs")]
    reg = RunRegistry(a.runs_root, a.runs)
    found = reg.discover()
    print(f"dashboard: {len(found)} run(s) at http://{a.host}:{a.port}/", flush=True)
    import uvicorn

    uvicorn.run(build_app(reg, a.static_dir), host=a.host, port=a.port, log_level=a.log_level)
    return 0


if __name__ == "__main__":
    sys.exit(main())
