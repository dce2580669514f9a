"""Any Hugging Face causal LM behind the trainer's model interface.

The reference trains whatever ``AutoModelForCausalLM`` loads
(trainer/model.py:496-524).  The native decoders here cover Qwen2 / Qwen3 /
Qwen3-MoE (sm_100a kernels) and DeepSeek-V4 (eager); every other
architecture whose ``config.json`` transformers knows (Llama, Mistral, Gemma,
Phi-3, GPT-2, ...) trains through this adapter: the transformers module runs
eagerly (packed documents through ``position_ids``, which transformers turns
into a block-causal mask; FlashAttention-2 varlen on the GPU when flash_attn
is installed, SDPA otherwise), while its parameters are views of one flat
store so the sharded AdamW, checkpoints, the chunked LM-head loss and the
policy exporters apply unchanged.  Autograd gradients are added into the
store's fp32 gradient buffer after each backward (``collect_cpu_grads``).

Rollouts for these models come from ``inference.hf_generator`` (the
module's own KV cache, the native generator's sampling semantics).  Not
supported with this adapter: tensor, expert and context parallelism, LoRA /
QLoRA, and heads the fused loss cannot express (an LM-head bias, logit
soft-capping or scaling).
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

import torch
from torch import nn

from .layers import BatchCtx
from .params import FlatParams, ParamSpec

NATIVE_MODEL_TYPES = ("qwen2", "qwen3", "qwen3_moe", "deepseek_v4")


class HFGenericConfig:
    """A transformers config (as its ``config.json`` dict) with the few shape
    fields the trainer's FLOP count and data paths read."""

    generic_hf = True
    arch = "hf"

    def __init__(self, d: dict[str, Any], source: str | None = None):
        if d.get("model_type") in NATIVE_MODEL_TYPES:
            raise ValueError(f"{d['model_type']} has a native decoder; use it")
        self.d = dict(d)
        self.source = source  # local directory with the weights, when loaded from one
        # vision-language models nest the decoder's shape under text_config
        self.is_vlm = isinstance(self.d.get("vision_config"), dict)
        text = self.d.get("text_config") if isinstance(self.d.get("text_config"), dict) else {}
        g = (lambda k, default=None: text.get(k, self.d.get(k, default))) if text else self.d.get
        self.vocab_size = int(g("vocab_size"))
        self.hidden_size = int(g("hidden_size") or g("n_embd") or g("d_model"))
        self.num_layers = int(g("num_hidden_layers") or g("n_layer") or g("num_layers"))
        self.num_heads = int(g("num_attention_heads") or g("n_head"))
        self.num_kv_heads = int(g("num_key_value_heads") or self.num_heads)
        self.head_dim = int(g("head_dim") or self.hidden_size // self.num_heads)
        self.intermediate_size = int(g("intermediate_size") or g("n_inner") or 4 * self.hidden_size)
        self.tie_embeddings = bool(g("tie_word_embeddings", True))
        self.num_experts = int(g("num_local_experts") or g("num_experts") or 0)
        self.num_experts_per_tok = int(g("num_experts_per_tok") or 0)
        self.moe_intermediate_size = int(g("moe_intermediate_size") or self.intermediate_size)
        self.max_position = int(g("max_position_embeddings") or g("n_positions") or 4096)
        self.q_dim = self.num_heads * self.head_dim
        self.kv_dim = self.num_kv_heads * self.head_dim
        self.qkv_dim = self.q_dim + 2 * self.kv_dim
        for key in ("final_logit_softcapping", "logit_scale"):
            if g(key) not in (None, 0, 1, 1.0):
                raise NotImplementedError(f"{key}={g(key)} is not expressible in the fused LM-head loss")

    @property
    def model_type(self) -> str:
        return self.d.get("model_type", "")

    def layer_is_moe(self, i: int) -> bool:
        return self.num_experts > 0

    def to_dict(self) -> dict[str, Any]:
        return dict(self.d)

    def to_hf_config(self) -> dict[str, Any]:
        return dict(self.d)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "HFGenericConfig":
        return cls(d)

    def transformers_config(self):
        from transformers import AutoConfig

        d = {k: v for k, v in self.d.items() if k not in ("architectures", "transformers_version", "torch_dtype")}
        return AutoConfig.for_model(**d)

    def image_tokens(self, grid_thw) -> int:
        """Placeholder tokens of one image of patch grid (t, h, w) after the
        vision tower's spatial merge."""
        merge = int((self.d.get("vision_config") or {}).get("spatial_merge_size", 1))
        t, h, w = (int(x) for x in grid_thw)
        return t * h * w // (merge * merge)


def _attn_impl(device: torch.device) -> str:
    if device.type == "cuda":
        try:
            import flash_attn  # noqa: F401

            return "flash_attention_2"
        except ImportError:
            pass
    return "sdpa"


class HFCausalLMTrainable:
    eager = True  # the engine collects autograd gradients after every backward

    def __init__(self, cfg: HFGenericConfig, device, dtype=None, dp_rank: int = 0, dp_world: int = 1, seed: int = 0,
                 init: bool = True, with_grad: bool = True, with_optimizer: bool = True):
        from transformers import AutoModelForCausalLM, AutoModelForImageTextToText

        self.cfg = cfg
        self.device = torch.device(device)
        dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        torch.manual_seed(seed)
        auto = AutoModelForImageTextToText if cfg.is_vlm else AutoModelForCausalLM
        with torch.device(self.device):
            module = auto.from_config(cfg.transformers_config(), attn_implementation=_attn_impl(self.device))
        self.module = module.to(dtype)
        self.module.train()
        out = self.module.get_output_embeddings()
        if out is None or getattr(out, "bias", None) is not None:
            raise NotImplementedError("the fused LM-head loss needs a bias-free linear output embedding")
        # one store entry per parameter object (tied weights share one entry)
        self._owners: dict[str, list[str]] = {}
        first: dict[int, str] = {}
        for n, p in self.module.named_parameters(remove_duplicate=False):
            key = first.setdefault(id(p), n)
            self._owners.setdefault(key, []).append(n)
        self._head_name = first[id(out.weight)]
        params = dict(self.module.named_parameters())
        specs = [ParamSpec(n, tuple(params[n].shape), weight_decay=params[n].dim() >= 2) for n in self._owners]
        self.flat = FlatParams(specs, self.device, dtype, dp_rank, dp_world, with_grad, with_optimizer)
        self.expert_flat = None
        self._bind(params)
        if cfg.source and init is False:
            self.load_pretrained(cfg.source)
        # trainer-interface attributes of the native models
        self.lora = None
        self.quant = None
        self.tp_size, self.tp_rank, self.tp_group, self.tp_fabric = 1, 0, None, None
        self.ep_size, self.ep_rank, self.ep_dp_rank, self.ep_group = 1, 0, 0, None
        self.fused_cpu = True

    def _bind(self, params: dict[str, nn.Parameter]) -> None:
        with torch.no_grad():
            for n in self._owners:
                self.flat.view(n).copy_(params[n].detach())
        self.flat.sync_master_from_compute()
        for n, names in self._owners.items():
            new = nn.Parameter(self.flat.view(n), requires_grad=params[n].requires_grad)
            for full in names:
                owner_name, _, leaf = full.rpartition(".")
                owner = self.module.get_submodule(owner_name) if owner_name else self.module
                setattr(owner, leaf, new)

    # ------------------------------------------------------ trainer interface
    @property
    def trainable(self) -> FlatParams:
        return self.flat

    @property
    def inv_freq(self):
        return None

    def batch_ctx(self, position_ids, cu_seqlens, max_seqlen, cp=None) -> BatchCtx:
        if cp is not None:
            raise NotImplementedError("Hugging Face models train without context parallelism here")
        return BatchCtx(pos=position_ids.reshape(-1).to(self.device), cu_seqlens=cu_seqlens.to(self.device),
                        max_seqlen=int(max_seqlen), inv_freq=None)

    def hidden(self, input_ids: torch.Tensor, batch: BatchCtx) -> torch.Tensor:
        """Final hidden states [T, H] of one packed row: per-document
        position ids make transformers mask across document boundaries."""
        if self.cfg.is_vlm:
            return self._hidden_vlm(input_ids, batch)
        ids = input_ids.reshape(1, -1).to(self.device)
        pos = batch.pos.reshape(1, -1).to(torch.int64)
        out = self.module.base_model(input_ids=ids, position_ids=pos, use_cache=False)
        h = out.last_hidden_state if hasattr(out, "last_hidden_state") else out[0]
        return h.reshape(ids.shape[1], -1)

    def _hidden_vlm(self, input_ids: torch.Tensor, batch: BatchCtx) -> torch.Tensor:
        """Vision-language models compute their own (multimodal rotary)
        positions from a document's tokens and image grids, so each document
        of the row runs on its own with its images (``doc_images`` of them,
        in order: pixel rows = t * h * w patches per image)."""
        ids = input_ids.reshape(-1).to(self.device)
        cu = batch.cu_seqlens.tolist()
        mm = batch.mm or {}
        pix, grid = mm.get("pixel_values"), mm.get("image_grid_thw")
        per_doc = mm.get("doc_images") or [0] * (len(cu) - 1)
        img_tok = self.cfg.d.get("image_token_id")
        outs, gi, pi = [], 0, 0
        for d in range(len(cu) - 1):
            doc = ids[cu[d]:cu[d + 1]]
            kw = {}
            k = int(per_doc[d])
            if k:
                g = grid[gi:gi + k]
                n = int(g.prod(-1).sum())
                want = sum(self.cfg.image_tokens(row) for row in g.tolist())
                if img_tok is not None and int((doc == img_tok).sum()) != want:
                    raise ValueError(f"document {d} has {int((doc == img_tok).sum())} image tokens for images "
                                     f"that need {want}")
                kw = {"pixel_values": pix[pi:pi + n].to(self.module.dtype), "image_grid_thw": g}
                gi, pi = gi + k, pi + n
            out = self.module.base_model(input_ids=doc[None], use_cache=False, **kw)
            h = out.last_hidden_state if hasattr(out, "last_hidden_state") else out[0]
            outs.append(h[0])
        return torch.cat(outs, 0)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return h @ self.head_weight().t()

    def head_weight(self) -> torch.Tensor:
        return self.flat.view(self._head_name)

    def head_grad(self) -> torch.Tensor | None:
        return self.flat.grad_view(self._head_name)

    def collect_cpu_grads(self) -> None:
        for n in self._owners:
            p = self.module.get_parameter(n)
            if p.grad is not None:
                g = self.flat.grad_view(n)
                if g is not None:
                    g.add_(p.grad.float())
                p.grad = None

    def finalize_grads(self) -> None:
        for name, _, _, _ in getattr(self, "_frozen", []):
            g = self.flat.grad_view(name)
            if g is not None:
                g.zero_()  # frozen parameters add nothing to the clip norm

    def freeze_prefix(self, prefix: str) -> int:
        """Freeze every parameter under the submodule ``prefix`` (e.g. the
        vision tower, ``model.visual``): it gets no gradient, and its values
        (bf16 and this rank's fp32 master part) are put back after every
        optimizer step, so weight decay does not move it either.  Returns how
        many parameters."""
        flat = self.flat
        lo, hi = flat.dp_rank * flat.shard_numel, (flat.dp_rank + 1) * flat.shard_numel
        self._frozen = getattr(self, "_frozen", [])
        for name, names in self._owners.items():
            if any(x == prefix or x.startswith(prefix + ".") for x in names):
                self.module.get_parameter(name).requires_grad_(False)
                off, k = flat.offsets[name]
                a, b = max(off, lo), min(off + k, hi)
                master = flat.master[a - lo:b - lo].clone() if (flat.master is not None and a < b) else None
                self._frozen.append((name, flat.view(name).clone(), (a - lo, b - lo) if a < b else None, master))
        if not self._frozen:
            raise ValueError(f"no parameters under {prefix!r} to freeze")
        return len(self._frozen)

    def after_optimizer_step(self) -> None:
        for name, val, span, master in getattr(self, "_frozen", []):
            self.flat.view(name).copy_(val)
            if span is not None and master is not None:
                self.flat.master[span[0]:span[1]].copy_(master)

    def set_activation_checkpointing(self, every: int | None) -> None:
        if every is None:
            self.module.gradient_checkpointing_disable()
        else:
            self.module.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": False})

    def enable_activation_offload(self, on: bool = True) -> None:
        if on:
            raise NotImplementedError("activation offload is not available for Hugging Face models here")

    def extra_state(self) -> dict[str, torch.Tensor]:
        return {}

    def load_extra_state(self, tensors: dict[str, torch.Tensor]) -> None:
        pass

    # ------------------------------------------------------ weights in HF layout
    def hf_state_dict(self) -> dict[str, torch.Tensor]:
        """Every parameter under its transformers name (a tied head once)."""
        return {n: self.flat.view(n) for n in self._owners}

    def load_pretrained(self, path: str | Path) -> None:
        """Load ``*.safetensors`` of a transformers checkpoint directory."""
        from safetensors.torch import load_file

        files = sorted(Path(path).glob("*.safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {path}")
        alias = {full: n for n, names in self._owners.items() for full in names}
        missing = set(self._owners)
        with torch.no_grad():
            for fp in files:
                for k, v in load_file(str(fp)).items():
                    n = alias.get(k)
                    if n is None:
                        continue
                    self.flat.view(n).copy_(v.to(self.device))
                    missing.discard(n)
        if missing:
            raise KeyError(f"{path} lacks {sorted(missing)[:5]} ({len(missing)} tensors)")
        self.flat.sync_master_from_compute()
