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

# orchestrator.custom_rollout_function: unset = the native generator, one of
# VERIFIER_ROLLOUT_FUNCTIONS = verifiers-package environments, any other
# "module.path:function" = a user rollout function (orchestrator.custom_rollout)
NATIVE_ROLLOUT_FUNCTION = "native"


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
        self.data_cfg = d
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
        self.model_cfg = cfg.model
        self.epoch = 0
        self.cursor = 0
        # orchestrator.curriculum: the sampler picks every prompt; gates admit scored groups
        cur = getattr(getattr(cfg, "orchestrator", None), "curriculum", None)
        self.curriculum = None
        if cur is not None:
            from .curriculum import Curriculum

            self.curriculum = Curriculum(cur, len(self.rows), self.seed, self.shuffle)

    def _tokenizer(self):
        if self.tok is None:
            from ..data.tokenizer import tokenizer_for

            self.tok = tokenizer_for(self.model_cfg)
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
                from ..data.sft import template_kwargs

                # the row's tool schemas and template arguments (data.tools_column / chat_template_kwargs_column)
                ids = tok.apply_chat_template(prompt, tokenize=True, add_generation_prompt=True,
                                              **template_kwargs(r, self.data_cfg))
                ids = ids["input_ids"] if isinstance(ids, dict) else ids
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
        if self.curriculum is not None:
            for _ in range(n):
                i, key = self.curriculum.next_record_index()
                rec = self._record(i)
                rec.metadata["task_key"] = key
                out.append(rec)
            return out
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
        sd = {"epoch": self.epoch, "cursor": self.cursor}
        if self.curriculum is not None:
            sd["curriculum"] = self.curriculum.state_dict()
        return sd

    def load_state_dict(self, sd: dict) -> None:
        self.epoch, self.cursor = int(sd["epoch"]), int(sd["cursor"])
        if self.curriculum is not None and "curriculum" in sd:
            self.curriculum.load_state_dict(sd["curriculum"])


class EnvironmentPromptSource:
    """Chat prompts from native environments (``wavelet_b200.environments``),
    mixed by ``ratio`` (orchestrator.envs): each draw picks the environment
    whose share of the prompts handed out so far is furthest below its ratio
    (deterministic weighted round robin), then that environment's next row in
    a seeded per-epoch shuffle.  The rollout metadata names the environment
    and carries the row, so the reward scorer can call the environment's
    reward."""

    def __init__(self, envs: list[tuple[Any, float]], model_name: str, seed: int = 0, rank: int = 0, world: int = 1,
                 tokenizer=None, split: str = "train", model_cfg=None):
        if not envs:
            raise ValueError("EnvironmentPromptSource needs at least one environment")
        self.envs = envs
        self.model_name = model_name
        self.model_cfg = model_cfg  # the model section: chat template / remote-code settings of the tokenizer
        self.tok = tokenizer
        self.seed, self.rank, self.world = seed, rank, world
        self.split = split
        self.drawn = [0] * len(envs)
        self.cursor = [0] * len(envs)
        self.epoch = [0] * len(envs)

    def _rows(self, i: int) -> list[dict[str, Any]]:
        env = self.envs[i][0]
        return env.examples if self.split == "train" else env.eval_examples

    def _order(self, i: int) -> list[int]:
        idx = list(range(len(self._rows(i))))
        random.Random((self.seed * 7919 + self.epoch[i]) * 31 + i).shuffle(idx)
        return idx[self.rank :: self.world] or idx

    def _tokenizer(self):
        if self.tok is None:
            from ..data.tokenizer import load_tokenizer, tokenizer_for

            self.tok = tokenizer_for(self.model_cfg) if self.model_cfg is not None else load_tokenizer(self.model_name)
        return self.tok

    def _pick(self) -> int:
        total = sum(self.drawn) + 1
        wsum = sum(w for _, w in self.envs)
        deficit = [w / wsum * total - d for (_, w), d in zip(self.envs, self.drawn)]
        return max(range(len(self.envs)), key=lambda i: (deficit[i], -i))

    def take(self, n: int) -> list[PromptRecord]:
        out = []
        for _ in range(n):
            i = self._pick()
            order = self._order(i)
            if self.cursor[i] >= len(order):
                self.epoch[i] += 1
                self.cursor[i] = 0
                order = self._order(i)
            row = self._rows(i)[order[self.cursor[i]]]
            self.cursor[i] += 1
            self.drawn[i] += 1
            env = self.envs[i][0]
            prompt = env.chat(row)
            tok = self._tokenizer()
            if hasattr(tok, "apply_chat_template"):
                ids = tok.apply_chat_template(prompt, tokenize=True, add_generation_prompt=True)
            else:
                ids = tok.encode("\n".join(m["content"] for m in prompt))
            target = [{"role": "assistant", "content": str(row["answer"])}] if row.get("answer") is not None else None
            md = {"env": env.name, "env_row": row, "task": row.get("task", env.name), "source": env.name}
            out.append(PromptRecord(list(map(int, ids)), prompt, target, md,
                                    str(row.get("example_id", f"{env.name}-{self.drawn[i]}"))))
        return out

    def state_dict(self) -> dict:
        return {"drawn": list(self.drawn), "cursor": list(self.cursor), "epoch": list(self.epoch)}

    def load_state_dict(self, sd: dict) -> None:
        self.drawn, self.cursor, self.epoch = list(sd["drawn"]), list(sd["cursor"]), list(sd["epoch"])
