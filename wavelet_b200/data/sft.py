"""SFT data pipeline: sources, normalisation, tokenisation with role loss
masks, packing and a resumable per-rank iterator.

Sources (``data.source``):
* ``local`` — ``.jsonl`` / ``.json`` / ``.parquet`` files (one or many);
* ``hf`` — ``datasets.load_dataset`` (offline cache only on this machine);
* ``fake`` — synthetic token ids (``fake_vocab_size``, ``fake_length``,
  ``fake_input_ids``), no tokenizer needed.

Records are prompt/completion pairs or chat ``messages``; the loss mask is set
per message role by ``data.loss_mask`` (assistant only by default), and off
for any message with ``step_loss_mask: 0``.  Packing:
``pad`` (one example per row, right padding) or ``cat`` (examples concatenated
into ``seq_len`` windows with sequence boundaries kept in ``cu_seqlens`` so
attention never crosses examples).

Parity: data/sft.py:25-994 of the reference (sources, mixing, chat templates,
role loss masks, pad/cat packing, stateful resume).
"""

from __future__ import annotations

import json
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

from ..trainer.engine import PackedBatch


@dataclass
class Sample:
    input_ids: list[int]
    loss_mask: list[int]
    source: str = "local"
    mm: dict | None = None  # processor fields of the sample's images (pre-tokenized multimodal rows)


# ------------------------------------------------------------------- sources
def _paths(v) -> list[Path]:
    return [Path(p) for p in (v if isinstance(v, list) else [v])]


def load_payloads(path: Path) -> list[dict[str, Any]]:
    if path.suffix == ".jsonl":
        return [json.loads(l) for l in path.read_text(encoding="utf-8").splitlines() if l.strip()]
    if path.suffix == ".json":
        data = json.loads(path.read_text(encoding="utf-8"))
        return data if isinstance(data, list) else [data]
    if path.suffix == ".parquet":
        import pyarrow.parquet as pq

        return pq.read_table(path).to_pylist()
    raise ValueError(f"unsupported data file {path} (use .jsonl, .json or .parquet)")


def _mix(groups: list[list[dict]], probs: list[float] | None, strategy: str, seed: int) -> list[dict]:
    if len(groups) == 1:
        return groups[0]
    if probs is None:
        return [r for g in groups for r in g]
    if len(probs) != len(groups):
        raise ValueError("probabilities must match the number of dataset groups")
    rng = random.Random(seed)
    iters = [list(g) for g in groups]
    pos = [0] * len(groups)
    out = []
    exhausted = set()
    while True:
        i = rng.choices(range(len(groups)), weights=probs)[0]
        if pos[i] >= len(iters[i]):
            exhausted.add(i)
            if strategy == "first_exhausted" or len(exhausted) == len(groups):
                break
            pos[i] = 0
        out.append(iters[i][pos[i]])
        pos[i] += 1
    return out


def load_records(cfg) -> list[dict[str, Any]]:
    if cfg.source == "local":
        groups = [load_payloads(p) for p in _paths(cfg.path)]
    elif cfg.source == "hf":
        from datasets import load_dataset  # offline cache only

        pairs = list(zip(cfg.hf_subsets or [None] * len(cfg.hf_splits or ["train"]), cfg.hf_splits or ["train"] * len(cfg.hf_subsets or [None])))
        groups = [[dict(r) for r in load_dataset(cfg.hf_name, s, split=sp)] for s, sp in pairs]
    else:
        return []
    for g, name in zip(groups, [str(p) for p in _paths(cfg.path)] if cfg.source == "local" else [cfg.hf_name] * len(groups)):
        for r in g:
            r.setdefault("__source", Path(name).stem if cfg.source == "local" else name)
    rows = _mix(groups, cfg.probabilities, cfg.stopping_strategy, cfg.seed)
    if cfg.max_examples is not None:
        rows = rows[: cfg.max_examples]
    return rows


# ------------------------------------------------------------- normalisation
def normalize_messages(row: dict[str, Any], cfg) -> list[dict[str, Any]]:
    if cfg.messages_column in row and row[cfg.messages_column]:
        msgs = row[cfg.messages_column]
        if isinstance(msgs, str):
            msgs = json.loads(msgs)
        msgs = [dict(m) for m in msgs]
    else:
        prompt = row.get(cfg.prompt_column)
        completion = row.get(cfg.completion_column)
        if prompt is None or completion is None:
            raise ValueError(f"record has neither '{cfg.messages_column}' nor '{cfg.prompt_column}'/'{cfg.completion_column}'")
        msgs = []
        msgs += prompt if isinstance(prompt, list) else [{"role": "user", "content": str(prompt)}]
        msgs += completion if isinstance(completion, list) else [{"role": "assistant", "content": str(completion)}]
    if cfg.merge_messages_thinking:
        for m in msgs:
            th = m.pop("reasoning_content", None) or m.pop("thinking", None)
            if th and m.get("role") == "assistant":
                m["content"] = f"<think>\n{th}\n</think>\n\n{m.get('content') or ''}"
    if cfg.system_prompt and not (msgs and msgs[0].get("role") == "system"):
        msgs = [{"role": "system", "content": cfg.system_prompt}] + msgs
    return _decode_tool_calls(msgs)


def _decode_tool_calls(msgs: list[dict[str, Any]]) -> list[dict[str, Any]]:
    """Tool-call ``arguments`` stored as JSON text become objects (chat
    templates render objects); text that is not JSON stays as it is."""
    out = []
    for m in msgs:
        calls = m.get("tool_calls")
        if not isinstance(calls, list):
            out.append(m)
            continue
        fixed = []
        for c in calls:
            fn = c.get("function") if isinstance(c, dict) else None
            if isinstance(fn, dict) and isinstance(fn.get("arguments"), str):
                try:
                    c = {**c, "function": {**fn, "arguments": json.loads(fn["arguments"])}}
                except json.JSONDecodeError:
                    pass
            fixed.append(c)
        out.append({**m, "tool_calls": fixed})
    return out


def template_kwargs(row: dict[str, Any], cfg) -> dict[str, Any]:
    """Chat-template arguments of a row: its tool schemas (``data.tools_column``)
    and extra template arguments such as ``enable_thinking``
    (``data.chat_template_kwargs_column``)."""
    out: dict[str, Any] = {}
    tools = row.get(getattr(cfg, "tools_column", "tools"))
    if isinstance(tools, str):
        tools = json.loads(tools)
    if tools is not None:
        if not isinstance(tools, list):
            raise ValueError("tools must be a list when provided.")
        out["tools"] = tools
    extra = row.get(getattr(cfg, "chat_template_kwargs_column", "chat_template_kwargs"))
    if isinstance(extra, str):
        extra = json.loads(extra)
    if extra is not None:
        if not isinstance(extra, dict):
            raise ValueError("chat_template_kwargs must be an object when provided.")
        out.update(extra)
    return out


def _role_trainable(role: str, lm) -> bool:
    return bool(getattr(lm, role, False)) if role in ("system", "user", "assistant", "tool") else False


def _trainable(m: dict[str, Any], lm) -> int:
    """The role's ``data.loss_mask`` setting, switched off for a message whose
    ``step_loss_mask`` is 0 (e.g. an intermediate tool-calling turn)."""
    if not _role_trainable(m["role"], lm):
        return 0
    return 0 if m.get("step_loss_mask", 1) in (0, False) else 1


def tokenize_messages(msgs: list[dict[str, Any]], tok, cfg, kwargs: dict[str, Any] | None = None) -> Sample:
    """Tokenise message by message so every token knows its role.

    With a template-capable tokenizer the rendered prefix of messages[:i+1]
    is diffed against messages[:i] (exact under incremental templates); the
    char tokenizer renders each message independently.  ``kwargs`` (tools,
    ``enable_thinking``, ...) go to every template call.
    """
    kw = dict(kwargs or {})
    ids: list[int] = []
    mask: list[int] = []
    if hasattr(tok, "render_message"):
        for m in msgs:
            t = tok.encode(tok.render_message(m["role"], str(m.get("content") or "")))
            head = len(tok.encode(tok.role_header(m["role"])))
            ids += t
            mask += [0] * head + [_trainable(m, cfg.loss_mask)] * (len(t) - head)  # the role tag is never trained
        ids.append(tok.eos_token_id)
        mask.append(_trainable(msgs[-1], cfg.loss_mask))
        return Sample(ids, mask)
    prev: list[int] = []
    for i, m in enumerate(msgs):
        cur = tok.apply_chat_template(msgs[: i + 1], tokenize=True, add_generation_prompt=False, **kw)
        if hasattr(cur, "input_ids"):
            cur = cur["input_ids"]
        cur = list(cur)
        if cur[: len(prev)] != prev:  # non-incremental template: fall back to suffix tokens
            common = 0
            while common < min(len(cur), len(prev)) and cur[common] == prev[common]:
                common += 1
            ids = ids[:common]
            mask = mask[:common]
            prev = prev[:common]
        new = cur[len(prev):]
        head = 0
        if m["role"] == "assistant" and _trainable(m, cfg.loss_mask):
            # the generation prompt (assistant header) belongs to the context, not the completion
            gen = tok.apply_chat_template(msgs[:i], tokenize=True, add_generation_prompt=True, **kw) if i else []
            if hasattr(gen, "input_ids"):
                gen = gen["input_ids"]
            gen = list(gen)
            if len(gen) >= len(prev) and gen[: len(prev)] == prev and cur[: len(gen)] == gen:
                head = len(gen) - len(prev)
        ids += new
        mask += [0] * head + [_trainable(m, cfg.loss_mask)] * (len(new) - head)
        prev = cur
    return Sample(ids, mask)


def _pretokenized(r: dict[str, Any]) -> Sample:
    """A row that is already token ids (``input_ids``, optional ``loss_mask``
    or ``labels`` with -100 for context) and optional ``mm_kwargs`` (the
    processor's image fields, image placeholder tokens already expanded)."""
    from .multimodal import as_mm_tensors

    ids = [int(t) for t in r["input_ids"]]
    if r.get("loss_mask") is not None:
        mask = [int(bool(x)) for x in r["loss_mask"]]
    elif r.get("labels") is not None:
        mask = [int(x != -100) for x in r["labels"]]
    else:
        mask = [1] * len(ids)
    if len(mask) != len(ids):
        raise ValueError("a pre-tokenized row needs one loss-mask entry per token")
    return Sample(ids, mask, mm=as_mm_tensors(r.get("mm_kwargs")))


def _check_fits(s: Sample, n: int) -> None:
    if s.mm and len(s.input_ids) > n:
        raise ValueError(f"a sample with image inputs has {len(s.input_ids)} tokens, more than the {n} of a row: "
                         "cutting it would split its image tokens from their pixels")


# ----------------------------------------------------------------- datasets
@dataclass
class SFTDataState:
    epoch: int = 0
    cursor: int = 0
    num_samples: dict[str, int] = field(default_factory=dict)
    num_tokens: dict[str, int] = field(default_factory=dict)


class SFTDataset:
    """Per-rank iterator of packed micro-batches with a resumable cursor."""

    def __init__(self, cfg, tokenizer=None, dp_rank: int = 0, dp_world: int = 1, seed: int = 0):
        self.cfg = cfg
        self.tok = tokenizer
        self.dp_rank = dp_rank
        self.dp_world = dp_world
        self.seed = seed + cfg.seed
        self.state = SFTDataState()
        self._samples: list[Sample] | None = None

    # samples --------------------------------------------------------------
    def _fake_samples(self) -> list[Sample]:
        c = self.cfg
        n = c.max_examples or max(c.batch_size * 4, 8)
        g = torch.Generator().manual_seed(self.seed)
        out = []
        lo, hi = getattr(c, "fake_prompt_fraction", (0.0, 0.0))
        for i in range(n):
            L = c.seq_len if c.fake_length == "fixed" else int(torch.randint(max(8, c.seq_len // 4), c.seq_len + 1, (1,), generator=g))
            if c.fake_input_ids == "increasing":
                ids = [(3 + i + j) % c.fake_vocab_size for j in range(L)]
            else:
                ids = torch.randint(3, c.fake_vocab_size, (L,), generator=g).tolist()
            f = lo + (hi - lo) * float(torch.rand((), generator=g)) if hi > 0 else 0.0
            mask = [0] * int(f * L) + [1] * (L - int(f * L))
            out.append(Sample(ids, mask, "fake"))
        return out

    def samples(self) -> list[Sample]:
        if self._samples is None:
            if self.cfg.source == "fake":
                self._samples = self._fake_samples()
            else:
                self._samples = []
                for r in load_records(self.cfg):
                    if "input_ids" in r:
                        s = _pretokenized(r)  # e.g. processor output of a vision-language sample
                    else:
                        if self.tok is None:
                            raise ValueError("a tokenizer is required for non-fake SFT data")
                        s = tokenize_messages(normalize_messages(r, self.cfg), self.tok, self.cfg,
                                              template_kwargs(r, self.cfg))
                    s.source = r.get("__source", "local")
                    if s.input_ids:
                        self._samples.append(s)
        return self._samples

    def _order(self, epoch: int) -> list[int]:
        idx = list(range(len(self.samples())))
        if self.cfg.shuffle:
            random.Random(self.seed * 7919 + epoch).shuffle(idx)
        return idx

    def _next_sample(self) -> Sample:
        order = self._order(self.state.epoch)
        if not order:
            raise ValueError("empty SFT dataset")
        while True:
            if self.state.cursor >= len(order):
                self.state.epoch += 1
                self.state.cursor = 0
                order = self._order(self.state.epoch)
            i = order[self.state.cursor]
            self.state.cursor += 1
            if (self.state.cursor - 1) % self.dp_world == self.dp_rank:
                s = self.samples()[i]
                self._last_index = i
                self.state.num_samples[s.source] = self.state.num_samples.get(s.source, 0) + 1
                self.state.num_tokens[s.source] = self.state.num_tokens.get(s.source, 0) + len(s.input_ids)
                return s

    # batches ---------------------------------------------------------------
    def next_micro_batch(self) -> PackedBatch:
        c = self.cfg
        S = c.seq_len
        mode = getattr(c, "pack_function", "pad")
        seqs, masks, mms = [], [], []
        if mode == "cat":
            budget = S * c.micro_batch_size
            used = 0
            while used < budget:
                # a sample that did not fit the previous window opens this one; it is
                # already past the cursor, so the state carries its index (resume)
                pend = getattr(self, "_pending_index", None)
                if pend is not None:
                    s, idx = self.samples()[pend], pend
                else:
                    s = self._next_sample()
                    idx = self._last_index
                self._pending_index = None
                take = min(len(s.input_ids), budget - used)
                if take < len(s.input_ids) and used > 0:
                    self._pending_index = idx
                    break
                _check_fits(s, take)
                seqs.append(torch.tensor(s.input_ids[:take]))
                masks.append(torch.tensor(s.loss_mask[:take], dtype=torch.float32))
                mms.append(s.mm)
                used += take
        else:
            for _ in range(c.micro_batch_size):
                s = self._next_sample()
                _check_fits(s, S)
                seqs.append(torch.tensor(s.input_ids[:S]))
                masks.append(torch.tensor(s.loss_mask[:S], dtype=torch.float32))
                mms.append(s.mm)
        return pack(seqs, masks, mms)

    def eval_batches(self, max_batches: int | None = None):
        """One ordered pass over this rank's share of the samples (validation)."""
        c = self.cfg
        mine = [s for i, s in enumerate(self.samples()) if i % self.dp_world == self.dp_rank]
        n = 0
        for i in range(0, len(mine), c.micro_batch_size):
            if max_batches is not None and n >= max_batches:
                return
            grp = mine[i : i + c.micro_batch_size]
            for s in grp:
                _check_fits(s, c.seq_len)
            yield pack([torch.tensor(s.input_ids[: c.seq_len]) for s in grp],
                       [torch.tensor(s.loss_mask[: c.seq_len], dtype=torch.float32) for s in grp],
                       [s.mm for s in grp])
            n += 1

    def state_dict(self) -> dict[str, Any]:
        return {"epoch": self.state.epoch, "cursor": self.state.cursor, "num_samples": dict(self.state.num_samples),
                "num_tokens": dict(self.state.num_tokens), "pending": getattr(self, "_pending_index", None)}

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        self.state = SFTDataState(int(sd["epoch"]), int(sd["cursor"]), dict(sd.get("num_samples", {})),
                                  dict(sd.get("num_tokens", {})))
        self._pending_index = sd.get("pending")


def pack(seqs: list[torch.Tensor], masks: list[torch.Tensor], mms: list | None = None) -> PackedBatch:
    """Concatenate sequences; target of position t is token t+1 of the same
    sequence (last position of each sequence is ignored).  ``mms``: the
    documents' image fields (``data.multimodal.pack_multimodal_row``)."""
    ids = torch.cat(seqs).long()
    lens = [len(s) for s in seqs]
    cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lens, dtype=torch.int32).cumsum(0)
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens])
    tg, mk = [], []
    for s, m in zip(seqs, masks):
        t = torch.full_like(s, -100, dtype=torch.long)
        t[:-1] = s[1:]
        # the loss mask marks trainable *target* tokens
        mm = torch.zeros(len(s), dtype=torch.float32)
        mm[:-1] = m[1:].float()
        tg.append(t)
        mk.append(mm)
    tgt = torch.cat(tg)
    mask = torch.cat(mk)
    tgt = torch.where(mask > 0, tgt, torch.full_like(tgt, -100))
    mm = None
    if mms is not None:
        from .multimodal import pack_multimodal_row

        mm = pack_multimodal_row(list(mms))
    return PackedBatch(ids, pos, cu, max(lens), tgt, mask, mm=mm)


class PrefetchingDataset:
    """``data.num_workers`` > 0: a background thread builds micro-batches
    ``depth`` ahead of the trainer (tokenised samples are packed and pinned
    while the GPU works).  ``state_dict`` is the state right after the last
    batch the trainer took, so a checkpoint never skips prefetched batches.
    Wrap a dataset after its state was restored."""

    def __init__(self, dataset, depth: int):
        import queue
        import threading

        self.dataset = dataset
        self._state = dataset.state_dict()
        self._q: "queue.Queue" = queue.Queue(maxsize=max(1, depth))
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._produce, name="wavelet-sft-prefetch", daemon=True)
        self._thread.start()

    def _produce(self) -> None:
        import queue

        while not self._stop.is_set():
            try:
                item = (self.dataset.next_micro_batch(), self.dataset.state_dict(), None)
            except BaseException as exc:  # noqa: BLE001 - raised in the trainer on its next take
                item = (None, None, exc)
            while not self._stop.is_set():
                try:
                    self._q.put(item, timeout=0.1)
                    break
                except queue.Full:
                    continue
            if item[2] is not None:
                return

    def next_micro_batch(self) -> PackedBatch:
        batch, state, exc = self._q.get()
        if exc is not None:
            raise exc
        self._state = state
        return batch

    def state_dict(self) -> dict[str, Any]:
        return self._state

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)

    def __getattr__(self, name: str):  # samples(), eval_batches(), ... of the wrapped dataset
        return getattr(self.dataset, name)
