"""Teacher log-probs for the distillation algorithms (reference
orchestrator/envs.py:1619-1760).

``algo.type: opd`` trains the policy towards a teacher by a reverse KL on
its own samples; ``opsd`` uses the policy itself as the teacher, conditioned
on a demonstration (a system turn rendered from ``algo.template`` with the
record's ``algo.demo_key`` metadata) placed before the rollout.  Both need the
teacher's log-prob of every trainable token of each rollout:

* ``opd``: the teacher is an inference server (``algo.teacher.base_url``;
  this framework's ``/score`` route: teacher-forced log-probs of a
  sequence's tokens after a prefix);
* ``opsd``: the rollout's own generator scores the prefixed sequences — the
  in-process model in integrated runs, the rollout servers' ``/score``
  otherwise.

The log-probs land in ``teacher_logprobs`` (one per trainable token, the
layout of ``inference_logprobs``).
"""

from __future__ import annotations

import json
import urllib.request
from dataclasses import replace
from typing import Any, Callable

import torch

from ..data.rl import RLExample

Scorer = Callable[[list[list[int]], list[int]], list[list[float]]]


def http_scorer(base_url: str, timeout_s: float = 120.0) -> Scorer:
    """A ``/score`` client of an inference server (``.../v1`` is accepted)."""
    root = base_url.rstrip("/")
    if root.endswith("/v1"):
        root = root[:-3]

    def score(seqs: list[list[int]], starts: list[int]) -> list[list[float]]:
        body = json.dumps({"sequences": seqs, "prompt_lens": starts, "temperature": 1.0}).encode()
        req = urllib.request.Request(root + "/score", data=body, headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=timeout_s) as r:
            return json.loads(r.read())["logprobs"]

    return score


def model_scorer(model) -> Scorer:
    """Teacher-forced log-probs from a model in this process."""
    from ..ops import lm_head

    @torch.no_grad()
    def score(seqs: list[list[int]], starts: list[int]) -> list[list[float]]:
        out = []
        for seq, st in zip(seqs, starts):
            ids = torch.tensor(seq, device=model.device)
            L = len(seq)
            ctx = model.batch_ctx(torch.arange(L, dtype=torch.int32), torch.tensor([0, L], dtype=torch.int32), L)
            h = model.hidden(ids, ctx)
            if h.is_cuda:
                lp, _ = lm_head.logprob_entropy(h[:-1], model.head_weight(), ids[1:], 1.0, want_entropy=False)
            else:
                lp, _ = lm_head.ref.logprob_entropy(model.logits(h[:-1]), ids[1:], 1.0)
            out.append(lp[st - 1:].float().tolist())
        return out

    return score


def opsd_prefix(record: RLExample, algo, tokenizer) -> list[int]:
    """Token ids of the demonstration turn placed before an OPSD rollout."""
    md = record.metadata or {}
    ex = md.get("verifier_example")
    demo = ex.get(algo.demo_key) if isinstance(ex, dict) else None
    if demo is None:
        demo = md.get(algo.demo_key)
    if demo is None:
        raise ValueError(f"OPSD needs {algo.demo_key!r} in the record's metadata")
    text = algo.template.format(demonstration=str(demo))
    if hasattr(tokenizer, "render_message"):
        return list(tokenizer.encode(tokenizer.render_message("system", text)))
    ids = tokenizer.apply_chat_template([{"role": "system", "content": text}], tokenize=True,
                                        add_generation_prompt=False)
    return list(ids["input_ids"] if isinstance(ids, dict) else ids)


def attach_teacher_logprobs(records: list[RLExample], cfg, scorer: Scorer | None = None,
                            tokenizer=None) -> list[RLExample]:
    """``records`` with ``teacher_logprobs`` for the distillation algorithms
    (unchanged for the others)."""
    from .algorithms import algorithm_loss_component

    if algorithm_loss_component(cfg.algo) != "ref_kl" or not records:
        return records
    opsd = cfg.algo.type == "opsd"
    if scorer is None:
        if opsd:
            raise ValueError("OPSD scoring needs the policy's scorer")
        t = cfg.algo.teacher
        scorer = http_scorer(t.base_url, t.timeout_seconds)
    if opsd and tokenizer is None:
        from ..data.tokenizer import tokenizer_for

        tokenizer = tokenizer_for(cfg.model)
    prefixes = [opsd_prefix(r, cfg.algo, tokenizer) if opsd else [] for r in records]
    for r in records:
        if r.input_ids is None or r.loss_mask is None:
            raise ValueError("distillation needs pretokenised rollouts (input_ids and loss_mask)")
        if r.loss_mask and r.loss_mask[0]:
            raise ValueError("the first token of a rollout cannot be trainable")
    lps = scorer([p + list(r.input_ids) for p, r in zip(prefixes, records)], [len(p) + 1 for p in prefixes])
    out = []
    for r, lp in zip(records, lps):
        # token i of the rollout sits at len(prefix) + i; its log-prob is lp[i - 1]
        out.append(replace(r, teacher_logprobs=[float(lp[i - 1]) for i, m in enumerate(r.loss_mask) if m]))
    return out


def scorer_for(cfg, engine: Any) -> Scorer | None:
    """The scorer of the distillation teacher: the OPD teacher server, or for
    OPSD the policy itself (its in-process model, else the rollout servers)."""
    if cfg.algo.type != "opsd":
        return None
    for e in (engine, getattr(engine, "engine", None)):  # the generator, or an engine behind an adapter
        model = getattr(e, "m", None) or getattr(e, "model", None)
        if model is not None and hasattr(model, "hidden"):
            return model_scorer(model)
    h = cfg.inference.http
    return http_scorer(f"http://{h.host}:{(h.ports or [h.port])[0]}")
