"""``wavelet convert-traces``: trace JSONL files (``<run>/traces/*.jsonl``) to
a dataset directory (reference tools/convert_traces.py).

Rows keep the standard trace columns (``format_version`` .. ``rollout_id``)
and put every other key into a JSON ``payload`` column, so heterogeneous
events share one schema.  Output: ``<output-dir>/<subset>/<split>-00000-of-00001.parquet``
plus ``dataset_info.json`` (loadable with ``datasets.load_dataset("parquet", ...)``).
``--repo-id`` (upload to the Hugging Face Hub) needs network access and is
rejected when ``HF_HUB_OFFLINE`` is set.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path
from typing import Any, Sequence

from ..orchestrator.trace import TRACE_FIELDS

REQUIRED = ("format_version", "timestamp", "subsystem", "event")


def trace_files(inputs: Sequence[Path]) -> list[Path]:
    files: set[Path] = set()
    for p in inputs:
        p = Path(p).expanduser()
        if p.is_file():
            files.add(p)
        elif p.is_dir():
            root = p / "traces" if (p / "traces").is_dir() else p
            files.update(x for x in root.rglob("*.jsonl") if x.is_file())
        else:
            raise FileNotFoundError(f"trace input not found: {p}")
    return sorted(files)


def load_rows(inputs: Sequence[Path], events: set[str] | None = None) -> list[dict[str, Any]]:
    rows = []
    for path in trace_files(inputs):
        for n, line in enumerate(path.read_text(encoding="utf-8").splitlines(), 1):
            if not line.strip():
                continue
            try:
                ev = json.loads(line)
            except json.JSONDecodeError as e:
                raise ValueError(f"invalid JSON in {path}:{n}: {e.msg}") from None
            missing = [k for k in REQUIRED if k not in ev]
            if missing:
                raise ValueError(f"{path}:{n} lacks trace fields {missing}")
            if events and ev["event"] not in events:
                continue
            row = {k: ev.get(k) for k in TRACE_FIELDS}
            for k in ("step", "queue_step", "optimizer_step", "policy_step"):
                row[k] = None if row[k] is None else int(row[k])
            for k in ("timestamp", "subsystem", "event", "task", "harness", "rollout_id"):
                row[k] = None if row[k] is None else str(row[k])
            row["payload"] = json.dumps({k: v for k, v in ev.items() if k not in TRACE_FIELDS}, sort_keys=True,
                                        default=str)
            row["source_file"] = str(path)
            rows.append(row)
    return rows


def write_dataset(rows: list[dict[str, Any]], output_dir: Path, subset: str, split: str) -> Path:
    import pyarrow as pa
    import pyarrow.parquet as pq

    d = Path(output_dir) / subset
    d.mkdir(parents=True, exist_ok=True)
    table = pa.Table.from_pylist(rows) if rows else pa.table({k: [] for k in (*TRACE_FIELDS, "payload")})
    path = d / f"{split}-00000-of-00001.parquet"
    pq.write_table(table, path)
    (Path(output_dir) / "dataset_info.json").write_text(json.dumps(
        {"subsets": {subset: {"splits": {split: {"num_rows": len(rows), "files": [str(path.name)]}}}},
         "columns": list(table.column_names)}, indent=2))
    return path


def main(argv: Sequence[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="wavelet convert-traces", description=__doc__)
    p.add_argument("inputs", nargs="+", type=Path, help="trace files, trace directories or run directories")
    dest = p.add_mutually_exclusive_group(required=True)
    dest.add_argument("--output-dir", type=Path, help="local dataset directory")
    dest.add_argument("--repo-id", help="Hugging Face dataset repository id")
    p.add_argument("--subset", default="default")
    p.add_argument("--split", default="train")
    p.add_argument("--event", action="append", default=[], help="keep only these event names (repeatable)")
    a = p.parse_args(sys.argv[1:] if argv is None else argv)
    rows = load_rows(a.inputs, set(a.event) or None)
    if a.repo_id:
        if os.environ.get("HF_HUB_OFFLINE"):
            raise SystemExit("--repo-id needs network access (HF_HUB_OFFLINE is set); use --output-dir")
        import tempfile

        from huggingface_hub import HfApi

        with tempfile.TemporaryDirectory() as tmp:
            write_dataset(rows, Path(tmp), a.subset, a.split)
            HfApi().upload_folder(folder_path=tmp, repo_id=a.repo_id, repo_type="dataset")
        print(f"uploaded {len(rows)} rows to {a.repo_id}")
        return 0
    path = write_dataset(rows, a.output_dir, a.subset, a.split)
    print(f"wrote {len(rows)} rows to {path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
