"""Prompt sources for the orchestrator (reference orchestrator/sources.py and
the dataset side of orchestrator/rollouts.py).

``FilePromptSource`` reads prompt rows from local JSONL / JSON / Parquet files
(``data.path``; several paths are mixed in order).  A row provides either
``prompt_ids`` (pretokenised) or ``prompt`` (a string or chat messages, which
needs the model's tokenizer), plus optional ``answer`` / ``target_completion``
(for ``reference_match`` rewards) and ``metadata``.  Rows are visited in a
seeded, epoch-reshuffled order; every data-parallel rank takes a disjoint
stride, and the cursor is part of the resumable state.
"""

from __future__ import annotations

import json
import random
from pathlib import Path
from typing import Any

from .rollouts import PromptRecord

# Names of rollout functions a config may select (orchestrator.custom_rollout_function)
NATIVE_ROLLOUT_FUNCTION = "native"
VERIFIER_ROLLOUT_FUNCTION = "verifiers"


def _read_rows(path: Path) -> list[dict[str, Any]]:
    if path.suffix == ".parquet":
        import pyarrow.parquet as pq

        return pq.read_table(path).to_pylist()
    text = path.read_text(encoding="utf-8")
    if path.suffix == ".json":
        data = json.loads(text)
        return data if isinstance(data, list) else [data]
    return [json.loads(l) for l in text.splitlines() if l.strip()]


def _as_messages(v) -> list[dict[str, str]]:
    if isinstance(v, str):
        return [{"role": "user", "content": v}]
    return list(v or [])


class FilePromptSource:
    def __init__(self, cfg, rank: int = 0, world: int = 1, tokenizer=None):
        d = cfg.data
        paths = d.path if isinstance(d.path, list) else [d.path]
        self.rows: list[dict[str, Any]] = []
        for p in paths:
            for r in _read_rows(Path(p)):
                r.setdefault("__source", Path(p).stem)
                self.rows.append(r)
        if not self.rows:
            raise ValueError(f"no prompt rows in {paths}")
        self.seed = int(getattr(d, "seed", 0))
        self.shuffle = bool(getattr(d, "shuffle", True))
        self.rank, self.world = rank, world
        self.tok = tokenizer
        self.model_name = cfg.model.name
        self.epoch = 0
        self.cursor = 0

    def _tokenizer(self):
        if self.tok is None:
            from ..data.tokenizer import load_tokenizer

            self.tok = load_tokenizer(self.model_name)
        return self.tok

    def _order(self) -> list[int]:
        idx = list(range(len(self.rows)))
        if self.shuffle:
            random.Random(self.seed * 7919 + self.epoch).shuffle(idx)
        return idx[self.rank :: self.world]

    def _record(self, i: int) -> PromptRecord:
        r = self.rows[i]
        prompt = _as_messages(r.get("prompt") or r.get("messages") or r.get("question"))
        ids = r.get("prompt_ids")
        if ids is None:
            tok = self._tokenizer()
            if hasattr(tok, "apply_chat_template") and prompt:
                ids = tok.apply_chat_template(prompt, tokenize=True, add_generation_prompt=True)
            else:
                ids = tok.encode(" ".join(m.get("content", "") for m in prompt))
        target = r.get("target_completion")
        if target is None and r.get("answer") is not None:
            target = [{"role": "assistant", "content": str(r["answer"])}]
        md = dict(r.get("metadata") or {})
        md.setdefault("source", r.get("__source"))
        if r.get("answer") is not None:
            md.setdefault("answer", r["answer"])
        return PromptRecord(list(map(int, ids)), prompt, target, md, str(r.get("id", r.get("example_id", i))))

    def take(self, n: int) -> list[PromptRecord]:
        out = []
        order = self._order()
        while len(out) < n:
            if self.cursor >= len(order):
                self.epoch += 1
                self.cursor = 0
                order = self._order()
            out.append(self._record(order[self.cursor]))
            self.cursor += 1
        return out

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "cursor": self.cursor}

    def load_state_dict(self, sd: dict) -> None:
        self.epoch, self.cursor = int(sd["epoch"]), int(sd["cursor"])
