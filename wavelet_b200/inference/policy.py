"""Inference engine interface and the in-process implementations.

``PolicyInferenceEngine`` (setup / load_policy / annotate / sleep / wake /
close) is the contract the orchestrator uses (inference/policy.py:75-100 of
the reference).  Implementations:

* ``PassthroughPolicyInferenceEngine`` — records already carry completions;
  only fills the default temperature;
* ``NativePolicyInferenceEngine`` — the native batched generator
  (``inference.engine.Generator``) in this process;
* ``HTTPPolicyInferenceEngine`` (``inference.client``) — one or more
  ``inference-server`` processes over HTTP.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import replace
from pathlib import Path
from typing import Any

from ..data.rl import RLExample


class PolicyInferenceEngine(ABC):
    # whether the engine serves several generation calls at once (HTTP servers
    # batch them) and can swap policy weights while generating
    concurrent_generate = False
    concurrent_policy_load = False

    def __init__(self, config):
        self.config = config
        self.policy_step: int | None = None

    @abstractmethod
    def setup(self) -> None: ...

    @abstractmethod
    def load_policy(self, policy_dir: Path, *, step: int) -> None: ...

    @abstractmethod
    def annotate(self, records: list[RLExample]) -> list[RLExample]: ...

    def close(self) -> None:
        pass

    def sleep(self) -> None:
        pass

    def wake(self, *, tags: list[str] | None = None) -> None:
        pass


class PassthroughPolicyInferenceEngine(PolicyInferenceEngine):
    def setup(self) -> None:
        pass

    def load_policy(self, policy_dir: Path, *, step: int) -> None:
        self.policy_step = step

    def annotate(self, records: list[RLExample]) -> list[RLExample]:
        t = self.config.inference.default_temperature
        return [r if r.temperatures is not None else replace(r, temperatures=t) for r in records]


def record_prompt_ids(r: RLExample, tokenizer=None) -> list[int]:
    md = r.metadata or {}
    if md.get("prompt_ids") is not None:
        return list(md["prompt_ids"])
    if r.input_ids is not None and r.loss_mask is not None and not any(r.loss_mask):
        return list(r.input_ids)
    if tokenizer is None:
        raise ValueError("record has no prompt token ids and no tokenizer is available")
    kw = dict(r.chat_template_kwargs or {})
    if r.tools:
        kw["tools"] = r.tools
    ids = tokenizer.apply_chat_template(r.prompt, tokenize=True, add_generation_prompt=True, **kw)
    return list(ids["input_ids"] if isinstance(ids, dict) else ids)


class NativePolicyInferenceEngine(PolicyInferenceEngine):
    """The native generator in this process (optionally sharing a model)."""

    def __init__(self, config, model=None, tokenizer=None):
        super().__init__(config)
        self.model = model
        self.tokenizer = tokenizer
        self.generator = None
        self.paused = False
        self.device_receiver = None  # transport.policy.DevicePolicyReceiver of a separate generator process

    def attach_device_receiver(self, index: int = 0):
        """Receive device policy updates (``policy_transfer.type: nccl``) in
        this generator process: announces the peer receive slots now so the
        trainer can find them."""
        from ..transport.policy import DevicePolicyReceiver

        self.device_receiver = DevicePolicyReceiver(self.model, self.config.output_dir, self.config.policy_transfer,
                                                    index)
        return self.device_receiver

    def setup(self) -> None:
        import torch

        from ..models.config import resolve_arch
        from ..models.qwen import build_model
        from .hf_generator import make_generator

        c = self.config
        if c.inference.vllm.tensor_parallel_size > 1 and self.model is None:
            raise NotImplementedError("inference.vllm.tensor_parallel_size > 1 runs as a torchrun group of "
                                      "inference-server processes (inference.tp_server), not in one process")
        if self.model is None:
            dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
            arch = resolve_arch(c.model.name, c.model.arch_overrides or None)
            self.model = build_model(arch, dev, seed=c.seed, with_grad=False, with_optimizer=False)
        v = c.inference.vllm
        self.generator = make_generator(self.model, max_num_seqs=v.max_num_seqs,
                                        max_model_len=v.max_model_len or c.data.seq_len,
                                        gpu_memory_utilization=v.gpu_memory_utilization, block_size=v.kv_block_size,
                                        cuda_graphs=v.cuda_graphs and not v.enforce_eager)

    def load_policy(self, policy_dir: Path, *, step: int) -> None:
        from ..transport.policy import load_policy_into

        if policy_dir is not None and Path(policy_dir).exists() and (Path(policy_dir) / "policy.json").exists():
            meta = load_policy_into(self.model, Path(policy_dir), self.device_receiver, step)
            step = int(meta.get("loaded_step", step))  # a peer update may already hold a newer step
        self.policy_step = step

    def close(self) -> None:
        if self.device_receiver is not None:
            self.device_receiver.close()
            self.device_receiver = None

    def sampling(self, overrides: dict[str, Any] | None = None):
        from .engine import SamplingParams

        s = self.config.inference.sampling
        p = SamplingParams(temperature=s.temperature if s.do_sample else 0.0, top_p=s.top_p, top_k=s.top_k,
                           min_p=s.min_p, max_tokens=s.max_completion_tokens or 256, min_tokens=s.min_tokens,
                           n=s.num_generations, seed=s.seed,
                           return_sampling_mask=self.config.sampling_mask_required())
        for k, v in (overrides or {}).items():
            if hasattr(p, k) and v is not None:
                setattr(p, k, v)
        return p

    def annotate(self, records: list[RLExample]) -> list[RLExample]:
        keep = self.config.inference.sampling.max_prompt_tokens
        prompts = [record_prompt_ids(r, self.tokenizer)[-keep:] if keep else record_prompt_ids(r, self.tokenizer)
                   for r in records]
        params = self.sampling()
        params.n = 1  # one completion per record
        comps = self.generator.generate(prompts, params)
        out = []
        for r, c in zip(records, comps):
            md = dict(r.metadata or {})
            md.update(prompt_ids=c.prompt_ids, completion_ids=c.token_ids, finish_reason=c.finish_reason,
                      completion_token_count=len(c.token_ids), prompt_token_count=len(c.prompt_ids), input_token_count=len(c.prompt_ids),
                      is_truncated=c.finish_reason == "length", policy_step=self.policy_step)
            text = self.tokenizer.decode(c.token_ids) if self.tokenizer is not None else ""
            out.append(replace(r, input_ids=c.prompt_ids + c.token_ids,
                               loss_mask=[False] * len(c.prompt_ids) + [True] * len(c.token_ids),
                               inference_logprobs=c.logprobs, temperatures=params.temperature,
                               sampling_mask=c.sampling_mask,
                               completion=[{"role": "assistant", "content": text}], metadata=md))
        return out

    def generate_ids(self, prompts: list[list[int]], overrides: dict[str, Any] | None = None):
        return self.generator.generate(prompts, self.sampling(overrides))

    def score(self, sequences: list[list[int]], prompt_lens: list[int], temperature: float = 1.0) -> list[list[float]]:
        """Teacher-forced log-probs of the completion part of each sequence."""
        import torch

        from ..ops import reference as ref

        m = self.model
        res = []
        with torch.no_grad():
            for seq, pl in zip(sequences, prompt_lens):
                ids = torch.tensor(seq, device=m.device)
                L = len(seq)
                ctx = m.batch_ctx(torch.arange(L, dtype=torch.int32), torch.tensor([0, L], dtype=torch.int32), L)
                h = m.hidden(ids, ctx)
                z = m.logits(h)
                lp, _ = ref.logprob_entropy(z[:-1], ids[1:], temperature)
                res.append(lp[pl - 1:].float().tolist())
        return res

    def sleep(self) -> None:
        if self.generator is not None:
            self.generator.release_cache()

    def wake(self, *, tags: list[str] | None = None) -> None:
        if self.generator is not None:
            self.generator.restore_cache()


def create_policy_inference_engine(config, model=None, tokenizer=None) -> PolicyInferenceEngine:
    mode = config.inference.mode
    if mode == "passthrough":
        return PassthroughPolicyInferenceEngine(config)
    if config.inference.vllm.server_backend == "offline":
        return NativePolicyInferenceEngine(config, model, tokenizer)
    from .client import HTTPPolicyInferenceEngine

    return HTTPPolicyInferenceEngine(config)
