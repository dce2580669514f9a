"""DeepSeek-V4 configuration (reference trainer/models/deepseek_v4/
configuration_deepseek_v4.py).

The field names, defaults and the config.json layout are those of the
published checkpoints (``model_type = "deepseek_v4"``), so configs load in
both directions.  Architecture knobs:

* residual stream of ``hc_mult`` parallel streams mixed by manifold-constrained
  hyper-connections (``hc_sinkhorn_iters``, ``hc_eps``);
* per-layer attention type (``layer_types``): ``sliding_attention``,
  ``compressed_sparse_attention`` (CSA: compressed entries chosen by a
  top-``index_topk`` indexer) or ``heavily_compressed_attention`` (HCA: all
  causally complete compressed entries), compression rates in
  ``compress_rates``; every type also reads a local ``sliding_window``;
* MoE with sqrt-softplus routing, ``num_hash_layers`` leading layers routed
  by a token-id table, clamped SwiGLU experts (``swiglu_limit``);
* two RoPE tables: ``main`` (``rope_theta``, sliding layers) and ``compress``
  (``compress_rope_theta`` plus optional YaRN scaling, compressed layers),
  applied to the trailing ``partial_rotary_factor`` of each head as
  interleaved channel pairs.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

LAYER_TYPES = ("sliding_attention", "compressed_sparse_attention", "heavily_compressed_attention")
CHECKPOINT_FORMAT = "deepseek_v4_native_v1"


class DeepseekV4Config:
    """Plain configuration object (no transformers dependency); unknown
    config.json keys are kept as attributes and written back."""

    model_type = "deepseek_v4"

    def __init__(self, vocab_size: int = 129280, hidden_size: int = 4096, moe_intermediate_size: int = 2048,
                 num_hidden_layers: int = 43, num_attention_heads: int = 64, num_key_value_heads: int = 1,
                 head_dim: int = 512, q_lora_rank: int = 1024, partial_rotary_factor: float | None = None,
                 qk_rope_head_dim: int | None = None, rope_theta: float = 10000.0,
                 compress_rope_theta: float = 160000.0, rope_parameters: dict | None = None,
                 rope_scaling: dict | None = None, max_position_embeddings: int = 1048576,
                 sliding_window: int = 128, o_groups: int = 8, o_lora_rank: int = 1024,
                 layer_types: list[str] | None = None, compress_rates: dict[str, int] | None = None,
                 index_n_heads: int = 64, index_head_dim: int = 128, index_topk: int = 512,
                 num_experts_per_tok: int = 6, n_routed_experts: int = 256, n_shared_experts: int = 1,
                 scoring_func: str = "sqrtsoftplus", topk_method: str = "noaux_tc", norm_topk_prob: bool = True,
                 routed_scaling_factor: float = 1.5, num_hash_layers: int = 3, swiglu_limit: float = 10.0,
                 hc_mult: int = 4, hc_sinkhorn_iters: int = 20, hc_eps: float = 1e-6, hidden_act: str = "silu",
                 initializer_range: float = 0.02, rms_norm_eps: float = 1e-6, use_cache: bool = True,
                 tie_word_embeddings: bool = False, attention_bias: bool = False, mlp_bias: bool = False,
                 attention_dropout: float = 0.0, output_router_logits: bool = False,
                 router_aux_loss_coef: float = 0.001, router_jitter_noise: float = 0.0,
                 pad_token_id: int | None = None, bos_token_id: int | None = 0, eos_token_id: Any = 1, **kwargs):
        legacy_ratios = kwargs.pop("compress_ratios", None)  # published per-layer 0 / CSA / HCA rate list
        kwargs.pop("mlp_layer_types", None)
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.moe_intermediate_size = moe_intermediate_size
        self.num_hidden_layers = num_hidden_layers
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = head_dim
        self.q_lora_rank = q_lora_rank
        if partial_rotary_factor is None:
            partial_rotary_factor = qk_rope_head_dim / head_dim if qk_rope_head_dim is not None else 64 / 512
        self.partial_rotary_factor = float(partial_rotary_factor)
        self.qk_rope_head_dim = int(head_dim * self.partial_rotary_factor)
        self.rope_theta = rope_theta
        self.compress_rope_theta = compress_rope_theta
        self.max_position_embeddings = max_position_embeddings
        self.sliding_window = sliding_window
        self.o_groups = o_groups
        self.o_lora_rank = o_lora_rank
        self.compress_rates = dict(compress_rates) if compress_rates is not None else {
            "compressed_sparse_attention": 4, "heavily_compressed_attention": 128}
        if layer_types is None and legacy_ratios is not None:
            by_rate = {0: "sliding_attention", **{r: t for t, r in self.compress_rates.items()}}
            layer_types = [by_rate[int(r)] for r in legacy_ratios[:num_hidden_layers]]
        if layer_types is None:  # two HCA layers, then CSA / HCA alternating
            layer_types = ["heavily_compressed_attention"] * min(num_hidden_layers, 2) + [
                "compressed_sparse_attention" if i % 2 else "heavily_compressed_attention"
                for i in range(max(num_hidden_layers - 2, 0))]
        self.layer_types = list(layer_types)
        self.compress_ratios = [self.compress_rates.get(t, 0) for t in self.layer_types]
        self.index_n_heads = index_n_heads
        self.index_head_dim = index_head_dim
        self.index_topk = index_topk
        self.num_experts_per_tok = num_experts_per_tok
        self.n_routed_experts = n_routed_experts
        self.n_shared_experts = n_shared_experts
        self.scoring_func = scoring_func
        self.topk_method = topk_method
        self.norm_topk_prob = norm_topk_prob
        self.routed_scaling_factor = routed_scaling_factor
        self.num_hash_layers = num_hash_layers
        self.swiglu_limit = swiglu_limit
        self.hc_mult = hc_mult
        self.hc_sinkhorn_iters = hc_sinkhorn_iters
        self.hc_eps = hc_eps
        self.hidden_act = hidden_act
        self.initializer_range = initializer_range
        self.rms_norm_eps = rms_norm_eps
        self.use_cache = use_cache
        self.attention_bias = attention_bias
        self.mlp_bias = mlp_bias
        self.attention_dropout = attention_dropout
        self.output_router_logits = output_router_logits
        self.router_aux_loss_coef = router_aux_loss_coef
        self.router_jitter_noise = router_jitter_noise
        self.pad_token_id = pad_token_id
        self.bos_token_id = bos_token_id
        self.eos_token_id = eos_token_id
        self.tie_word_embeddings = tie_word_embeddings
        self._extra = dict(kwargs)
        for k, v in kwargs.items():
            setattr(self, k, v)
        self.rope_parameters = self._rope_tables(rope_parameters if rope_parameters is not None else rope_scaling)
        self.check_architecture()

    def set_extra(self, key: str, value: Any) -> None:
        """Set a field outside the architecture (written to config.json);
        ``None`` removes it."""
        if value is None:
            self._extra.pop(key, None)
            if hasattr(self, key):
                delattr(self, key)
            return
        self._extra[key] = value
        setattr(self, key, value)

    # aliases read by expert-parallel / shared-expert code
    @property
    def num_local_experts(self) -> int:
        return self.n_routed_experts

    @property
    def intermediate_size(self) -> int:
        return self.moe_intermediate_size

    def _rope_tables(self, raw: dict | None) -> dict[str, dict]:
        """``{"main": ..., "compress": ...}``; a flat dict (the published
        ``rope_scaling``) scales the compress table only."""
        raw = dict(raw or {})
        if isinstance(raw.get("main"), dict) and isinstance(raw.get("compress"), dict):
            return {"main": dict(raw["main"]), "compress": dict(raw["compress"])}
        flat = {k: v for k, v in raw.items() if k not in ("main", "compress")}
        kind = flat.pop("rope_type", flat.pop("type", "default"))
        compress = {**flat, "rope_type": kind, "rope_theta": self.compress_rope_theta,
                    "partial_rotary_factor": self.partial_rotary_factor}
        if kind == "yarn":
            compress.setdefault("attention_factor", 1.0)  # cos/sin are not rescaled by YaRN's mscale
        main = {"rope_type": "default", "rope_theta": self.rope_theta,
                "partial_rotary_factor": self.partial_rotary_factor}
        return {"main": main, "compress": compress}

    def check_architecture(self) -> None:
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError(f"layer_types has {len(self.layer_types)} entries for {self.num_hidden_layers} layers")
        bad = sorted(set(self.layer_types) - set(LAYER_TYPES))
        if bad:
            raise ValueError(f"layer_types entries must be one of {LAYER_TYPES}; got {bad}")
        for t in set(self.layer_types) - {"sliding_attention"}:
            if t not in self.compress_rates:
                raise ValueError(f"compress_rates is missing a rate for layer type {t!r}")
        if not 0 <= self.num_hash_layers <= self.num_hidden_layers:
            raise ValueError("num_hash_layers must be between 0 and num_hidden_layers")
        if self.qk_rope_head_dim % 2 or self.qk_rope_head_dim > self.head_dim:
            raise ValueError("the rotary part of a head must be an even number of channels within head_dim")
        if (self.num_attention_heads * self.head_dim) % self.o_groups:
            raise ValueError("o_groups must divide num_attention_heads * head_dim")

    # ---------------------------------------------------------------- files
    _FIELDS = ("vocab_size", "hidden_size", "moe_intermediate_size", "num_hidden_layers", "num_attention_heads",
               "num_key_value_heads", "head_dim", "q_lora_rank", "partial_rotary_factor", "qk_rope_head_dim",
               "rope_theta", "compress_rope_theta", "rope_parameters", "max_position_embeddings", "sliding_window",
               "o_groups", "o_lora_rank", "layer_types", "compress_rates", "compress_ratios", "index_n_heads",
               "index_head_dim", "index_topk", "num_experts_per_tok", "n_routed_experts", "n_shared_experts",
               "scoring_func", "topk_method", "norm_topk_prob", "routed_scaling_factor", "num_hash_layers",
               "swiglu_limit", "hc_mult", "hc_sinkhorn_iters", "hc_eps", "hidden_act", "initializer_range",
               "rms_norm_eps", "use_cache", "tie_word_embeddings", "attention_bias", "mlp_bias",
               "attention_dropout", "output_router_logits", "router_aux_loss_coef", "router_jitter_noise",
               "pad_token_id", "bos_token_id", "eos_token_id")

    def to_dict(self) -> dict[str, Any]:
        out = {k: getattr(self, k) for k in self._FIELDS}
        out.update({k: getattr(self, k) for k in self._extra})
        out["model_type"] = self.model_type
        return out

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "DeepseekV4Config":
        d = {k: v for k, v in d.items() if k not in ("model_type", "compress_ratios", "qk_rope_head_dim")
             or (k == "compress_ratios" and "layer_types" not in d)}
        return cls(**d)

    def save_pretrained(self, path: str | Path) -> None:
        p = Path(path)
        p.mkdir(parents=True, exist_ok=True)
        (p / "config.json").write_text(json.dumps(self.to_dict(), indent=2, sort_keys=True) + "\n")

    @classmethod
    def from_pretrained(cls, path: str | Path, **_: Any) -> "DeepseekV4Config":
        return cls.from_dict(json.loads((Path(path) / "config.json").read_text()))
