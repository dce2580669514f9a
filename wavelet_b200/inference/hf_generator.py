"""Generation for models trained through the transformers module adapter
(``models.hf_generic``): architectures without a native decoder.

The reference generates rollouts for any architecture with vLLM; here the
native paged-KV generator (``inference.engine.Generator``) covers the Qwen
decoders, and this generator covers the rest with the module's own KV cache:
prompts of one call are left-padded into batches of up to ``max_num_seqs``
rows, prefilled once and decoded a token at a time.  Sampling follows the
native generator exactly — temperature (0 = greedy at scale 1), top-k /
top-p thresholds on the raw logits, min-p on the scaled ones, the log-prob of
the sampled token under the processed distribution, the kept-token mask when
``return_sampling_mask`` asks for it, ``min_tokens`` before stop tokens, and
one seed per call — so the same ``SamplingParams`` mean the same thing for
both.  The module reads its parameters from the trainer's flat store, so an
integrated run generates with the weights of the latest optimizer step.
"""

from __future__ import annotations

import math
import time

import torch

from .engine import Completion, SamplingParams, sampling_thresholds_reference


class HFGenerator:
    def __init__(self, model, *, max_num_seqs: int = 64, max_model_len: int = 4096, **_ignored):
        self.m = model
        self.module = model.module
        self.dev = model.device
        self.max_num_seqs = max(1, int(max_num_seqs))
        self.max_model_len = int(max_model_len)
        self.stats: dict[str, float] = {}
        self.num_blocks = 0

    def kv_usage(self) -> float:
        return 0.0

    def release_cache(self) -> None:
        if self.dev.type == "cuda":
            torch.cuda.empty_cache()

    def restore_cache(self) -> None:
        pass

    # ------------------------------------------------------------ sampling
    def _sample(self, z: torch.Tensor, p: SamplingParams, g: torch.Generator):
        B = z.shape[0]
        zf = z.float()
        greedy = p.temperature <= 0
        inv = 1.0 if greedy else 1.0 / p.temperature
        zt = zf * inv
        thresh = None
        if p.top_k > 0 or p.top_p < 1.0:
            thresh = sampling_thresholds_reference(zf, [p.top_k] * B, [p.top_p] * B,
                                                   torch.full((B,), 0.0 if greedy else inv, device=z.device))
            zt = zt.masked_fill(zf < thresh[:, None], float("-inf"))
        if p.min_p > 0:
            zt = zt.masked_fill(zt < zt.max(-1, keepdim=True).values + math.log(p.min_p), float("-inf"))
        logp = torch.log_softmax(zt, -1)
        if greedy:
            tok = zt.argmax(-1)
        else:
            tok = torch.multinomial(logp.exp(), 1, generator=g)[:, 0]
        lp = logp.gather(1, tok[:, None])[:, 0]
        masks = None
        if p.truncated and p.return_sampling_mask:
            keep = torch.isfinite(zt)
            masks = [row.nonzero()[:, 0].tolist() for row in keep.cpu()]
        return tok, lp, masks

    # ------------------------------------------------------------ driver
    @torch.no_grad()
    def generate(self, prompts: list[list[int]], params: SamplingParams) -> list[Completion]:
        t0 = time.perf_counter()
        seed = params.seed if params.seed is not None else int(time.time_ns() & 0x7FFFFFFF)
        g = torch.Generator(device=self.dev if self.dev.type == "cuda" else "cpu").manual_seed(int(seed))
        rows = [(pi, si) for pi in range(len(prompts)) for si in range(params.n)]
        out: list[Completion] = []
        gen_tokens = 0
        for c0 in range(0, len(rows), self.max_num_seqs):
            chunk = rows[c0:c0 + self.max_num_seqs]
            outs, n = self._run(prompts, chunk, params, g)
            out += outs
            gen_tokens += n
        dt = time.perf_counter() - t0
        self.stats = {"generate_seconds": dt, "generated_tokens": float(gen_tokens),
                      "tokens_per_second": gen_tokens / dt if dt > 0 else 0.0}
        return out

    def _run(self, prompts, chunk, p: SamplingParams, g):
        ids_list = [prompts[pi] for pi, _ in chunk]
        B = len(chunk)
        L = max(len(x) for x in ids_list)
        budget = max(0, min(p.max_tokens, self.max_model_len - L))
        ids = torch.zeros(B, L, dtype=torch.long)
        am = torch.zeros(B, L, dtype=torch.long)
        for i, x in enumerate(ids_list):  # left padding: every row's last prompt token in the last column
            ids[i, L - len(x):] = torch.tensor(x, dtype=torch.long)
            am[i, L - len(x):] = 1
        ids, am = ids.to(self.dev), am.to(self.dev)
        pos = (am.cumsum(-1) - 1).clamp_min(0)
        res = self.module(input_ids=ids, attention_mask=am, position_ids=pos, use_cache=True)
        past = res.past_key_values
        z = res.logits[:, -1]
        toks: list[list[int]] = [[] for _ in range(B)]
        lps: list[list[float]] = [[] for _ in range(B)]
        masks: list[list[list[int]] | None] = [[] if (p.truncated and p.return_sampling_mask) else None
                                                for _ in range(B)]
        done = [None] * B
        last = pos[:, -1]
        stop = set(p.stop_token_ids)
        for k in range(budget):
            tok, lp, mk = self._sample(z, p, g)
            th, lh = tok.tolist(), lp.tolist()
            for i in range(B):
                if done[i] is not None:
                    continue
                toks[i].append(th[i])
                lps[i].append(lh[i])
                if masks[i] is not None:
                    masks[i].append(mk[i])
                if len(toks[i]) > p.min_tokens and th[i] in stop:
                    done[i] = "stop"
                elif len(toks[i]) >= budget:
                    done[i] = "length"
            if all(d is not None for d in done):
                break
            am = torch.cat([am, torch.ones(B, 1, dtype=am.dtype, device=self.dev)], 1)
            last = last + 1
            res = self.module(input_ids=tok[:, None], attention_mask=am, position_ids=last[:, None],
                              past_key_values=past, use_cache=True)
            past = res.past_key_values
            z = res.logits[:, -1]
        out = []
        for i, (pi, si) in enumerate(chunk):
            out.append(Completion(prompt_index=pi, sample_index=si, prompt_ids=list(prompts[pi]), token_ids=toks[i],
                                  logprobs=lps[i], finish_reason=done[i] or "length",
                                  sampling_mask=masks[i]))
        return out, sum(len(t) for t in toks)


def make_generator(model, **kw):
    """The native paged-KV generator for native decoders, ``HFGenerator`` for
    models that run through the transformers module."""
    if getattr(model.cfg, "generic_hf", False):
        return HFGenerator(model, **kw)
    from .engine import Generator

    return Generator(model, **kw)
