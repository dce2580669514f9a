"""Decoder architecture configurations (Qwen2 / Qwen3 dense, Qwen3-MoE).

The reference loads these architectures through Hugging Face
(``AutoModelForCausalLM`` in trainer/model.py:536); this framework implements
them natively.  ``from_hf_config`` accepts a Hugging Face ``config.json`` dict
so checkpoints and configs interoperate; ``PRESETS`` hold the shapes used by
the benchmarks (random init, no download).
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path
from typing import Any


@dataclass(frozen=True)
class ArchConfig:
    arch: str = "qwen3"  # qwen2 | qwen3 | qwen3_moe
    vocab_size: int = 151936
    hidden_size: int = 1024
    num_layers: int = 28
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    tie_embeddings: bool = True
    qkv_bias: bool = False
    qk_norm: bool = True
    max_position: int = 40960
    # MoE (arch == qwen3_moe)
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    router_aux_loss_coef: float = 0.001
    decoder_sparse_step: int = 1
    mlp_only_layers: tuple[int, ...] = field(default_factory=tuple)
    init_std: float = 0.02

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_is_moe(self, i: int) -> bool:
        return (
            self.is_moe
            and i not in self.mlp_only_layers
            and (i + 1) % max(1, self.decoder_sparse_step) == 0
        )

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def num_params(self, active_only: bool = False) -> int:
        H, I = self.hidden_size, self.intermediate_size
        attn = H * self.qkv_dim + self.q_dim * H + (self.qkv_dim if self.qkv_bias else 0)
        attn += 2 * H + (2 * self.head_dim if self.qk_norm else 0)
        total = 0
        for i in range(self.num_layers):
            if self.layer_is_moe(i):
                e = self.num_experts_per_tok if active_only else self.num_experts
                mlp = e * 3 * H * self.moe_intermediate_size + self.num_experts * H
            else:
                mlp = 3 * H * I
            total += attn + mlp
        emb = self.vocab_size * H
        total += emb + H + (0 if self.tie_embeddings else emb)
        return total

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "ArchConfig":
        d = dict(d)
        if "mlp_only_layers" in d:
            d["mlp_only_layers"] = tuple(d["mlp_only_layers"])
        known = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in d.items() if k in known})

    def to_dict(self) -> dict[str, Any]:
        d = asdict(self)
        d["mlp_only_layers"] = list(self.mlp_only_layers)
        return d

    def to_hf_config(self) -> dict[str, Any]:
        base = {
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate_size,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_eps,
            "tie_word_embeddings": self.tie_embeddings,
            "max_position_embeddings": self.max_position,
            "hidden_act": "silu",
            "torch_dtype": "bfloat16",
        }
        if self.arch == "qwen2":
            base.update(model_type="qwen2", architectures=["Qwen2ForCausalLM"])
        elif self.arch == "qwen3":
            base.update(model_type="qwen3", architectures=["Qwen3ForCausalLM"])
        else:
            base.update(
                model_type="qwen3_moe",
                architectures=["Qwen3MoeForCausalLM"],
                num_experts=self.num_experts,
                num_experts_per_tok=self.num_experts_per_tok,
                moe_intermediate_size=self.moe_intermediate_size,
                norm_topk_prob=self.norm_topk_prob,
                router_aux_loss_coef=self.router_aux_loss_coef,
                decoder_sparse_step=self.decoder_sparse_step,
                mlp_only_layers=list(self.mlp_only_layers),
            )
        return base


def from_hf_config(d: dict[str, Any]) -> ArchConfig:
    mt = d.get("model_type", "qwen3")
    arch = {"qwen2": "qwen2", "qwen3": "qwen3", "qwen3_moe": "qwen3_moe"}.get(mt)
    if arch is None:
        raise ValueError(f"unsupported model_type {mt!r} (supported: qwen2, qwen3, qwen3_moe)")
    H = d["hidden_size"]
    nh = d["num_attention_heads"]
    return ArchConfig(
        arch=arch,
        vocab_size=d["vocab_size"],
        hidden_size=H,
        num_layers=d["num_hidden_layers"],
        num_heads=nh,
        num_kv_heads=d.get("num_key_value_heads", nh),
        head_dim=d.get("head_dim") or H // nh,
        intermediate_size=d.get("intermediate_size", 4 * H),
        rope_theta=float(d.get("rope_theta", 1e6)),
        rms_eps=float(d.get("rms_norm_eps", 1e-6)),
        tie_embeddings=bool(d.get("tie_word_embeddings", False)),
        qkv_bias=arch == "qwen2",
        qk_norm=arch in ("qwen3", "qwen3_moe"),
        max_position=d.get("max_position_embeddings", 32768),
        num_experts=d.get("num_experts", 0) if arch == "qwen3_moe" else 0,
        num_experts_per_tok=d.get("num_experts_per_tok", 0) if arch == "qwen3_moe" else 0,
        moe_intermediate_size=d.get("moe_intermediate_size", 0) if arch == "qwen3_moe" else 0,
        norm_topk_prob=bool(d.get("norm_topk_prob", True)),
        router_aux_loss_coef=float(d.get("router_aux_loss_coef", 0.001)),
        decoder_sparse_step=int(d.get("decoder_sparse_step", 1)),
        mlp_only_layers=tuple(d.get("mlp_only_layers", []) or []),
    )


PRESETS: dict[str, ArchConfig] = {
    # Qwen2.5-7B shape (SFT / QLoRA benchmarks)
    "qwen2.5-7b": ArchConfig(
        arch="qwen2", vocab_size=152064, hidden_size=3584, num_layers=28, num_heads=28,
        num_kv_heads=4, head_dim=128, intermediate_size=18944, rope_theta=1e6,
        tie_embeddings=False, qkv_bias=True, qk_norm=False, max_position=32768,
    ),
    # Qwen3-4B shape (dense GRPO benchmark)
    "qwen3-4b": ArchConfig(
        arch="qwen3", vocab_size=151936, hidden_size=2560, num_layers=36, num_heads=32,
        num_kv_heads=8, head_dim=128, intermediate_size=9728, rope_theta=1e6,
        tie_embeddings=True, qkv_bias=False, qk_norm=True,
    ),
    # Qwen3-30B-A3B shape (MoE GRPO benchmark)
    "qwen3-30b-a3b": ArchConfig(
        arch="qwen3_moe", vocab_size=151936, hidden_size=2048, num_layers=48, num_heads=32,
        num_kv_heads=4, head_dim=128, intermediate_size=6144, rope_theta=1e6,
        tie_embeddings=False, qkv_bias=False, qk_norm=True, num_experts=128,
        num_experts_per_tok=8, moe_intermediate_size=768,
    ),
    # Qwen3-0.6B shape (the reference's own benchmark workload)
    "qwen3-0.6b": ArchConfig(
        arch="qwen3", vocab_size=151936, hidden_size=1024, num_layers=28, num_heads=16,
        num_kv_heads=8, head_dim=128, intermediate_size=3072, tie_embeddings=True,
    ),
    # Tiny decoder of the CPU/gloo plumbing configuration.  head_dim 32 keeps
    # it on the CPU reference path (the GPU kernels are specialised to 128).
    "tiny": ArchConfig(
        arch="qwen3", vocab_size=1024, hidden_size=128, num_layers=2, num_heads=4,
        num_kv_heads=2, head_dim=32, intermediate_size=512, rope_theta=1e4,
        tie_embeddings=False, qk_norm=False, max_position=4096,
    ),
    # Small GPU-kernel-compatible shapes for tests (head_dim 128).
    "tiny-gpu": ArchConfig(
        arch="qwen3", vocab_size=2048, hidden_size=256, num_layers=2, num_heads=4,
        num_kv_heads=2, head_dim=128, intermediate_size=512, rope_theta=1e4,
        tie_embeddings=False, qk_norm=True, max_position=4096,
    ),
    "tiny-qwen2-gpu": ArchConfig(
        arch="qwen2", vocab_size=2048, hidden_size=256, num_layers=2, num_heads=4,
        num_kv_heads=2, head_dim=128, intermediate_size=512, rope_theta=1e4,
        tie_embeddings=False, qkv_bias=True, qk_norm=False, max_position=4096,
    ),
    "tiny-moe-gpu": ArchConfig(
        arch="qwen3_moe", vocab_size=2048, hidden_size=256, num_layers=2, num_heads=4,
        num_kv_heads=2, head_dim=128, intermediate_size=512, rope_theta=1e4,
        tie_embeddings=False, qk_norm=True, num_experts=8, num_experts_per_tok=2,
        moe_intermediate_size=256, max_position=4096,
    ),
    "tiny-moe": ArchConfig(
        arch="qwen3_moe", vocab_size=1024, hidden_size=128, num_layers=2, num_heads=4,
        num_kv_heads=2, head_dim=32, intermediate_size=512, rope_theta=1e4,
        tie_embeddings=False, qk_norm=True, num_experts=8, num_experts_per_tok=2,
        moe_intermediate_size=64, max_position=4096,
    ),
}

# Names that the reference's configs use for the same shapes.
ALIASES = {
    "Qwen/Qwen2.5-7B": "qwen2.5-7b",
    "Qwen/Qwen2.5-7B-Instruct": "qwen2.5-7b",
    "Qwen/Qwen3-4B": "qwen3-4b",
    "Qwen/Qwen3-4B-Instruct-2507": "qwen3-4b",
    "Qwen/Qwen3-30B-A3B": "qwen3-30b-a3b",
    "Qwen/Qwen3-30B-A3B-Instruct-2507": "qwen3-30b-a3b",
    "Qwen/Qwen3-0.6B": "qwen3-0.6b",
}


# a DeepSeek-V4 of every attention type in three layers (CPU tests, smoke runs)
TINY_DEEPSEEK_V4 = dict(
    vocab_size=1024, hidden_size=64, num_hidden_layers=3, num_attention_heads=4, head_dim=32, q_lora_rank=32,
    partial_rotary_factor=0.5,
    layer_types=["sliding_attention", "compressed_sparse_attention", "heavily_compressed_attention"],
    compress_rates={"compressed_sparse_attention": 4, "heavily_compressed_attention": 16}, sliding_window=16,
    o_groups=2, o_lora_rank=16, index_n_heads=2, index_head_dim=32, index_topk=4, moe_intermediate_size=64,
    n_routed_experts=4, num_experts_per_tok=2, num_hash_layers=1, hc_mult=2, max_position_embeddings=4096)


# Small transformers configs of architectures without a native decoder (the
# generic Hugging Face path, models/hf_generic.py).
GENERIC_PRESETS: dict[str, dict[str, Any]] = {
    "tiny-llama": dict(model_type="llama", vocab_size=1024, hidden_size=128, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, intermediate_size=256,
                       max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=10000.0,
                       tie_word_embeddings=False),
    "tiny-mistral": dict(model_type="mistral", vocab_size=1024, hidden_size=128, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, intermediate_size=256,
                         max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=10000.0,
                         tie_word_embeddings=True, sliding_window=None),
    # a vision-language model (Qwen2.5-VL layout): 14-pixel patches, 2x2 merge
    "tiny-qwen2.5-vl": dict(
        model_type="qwen2_5_vl", image_token_id=1000, video_token_id=1001, vision_start_token_id=1002,
        vision_end_token_id=1003, tie_word_embeddings=False,
        text_config=dict(vocab_size=1024, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                         num_key_value_heads=2, intermediate_size=256, max_position_embeddings=4096,
                         rope_scaling={"type": "mrope", "mrope_section": [4, 6, 6]}),
        vision_config=dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, out_hidden_size=128,
                           patch_size=14, spatial_merge_size=2, temporal_patch_size=2, in_channels=3)),
}


def resolve_arch(name: str, overrides: dict[str, Any] | None = None) -> ArchConfig:
    """Resolve a model name: preset, alias, a local HF dir, or a config.json
    path.  A config.json of an architecture without a native decoder gives an
    ``HFGenericConfig`` (trained through the transformers module)."""
    key = ALIASES.get(name, name)
    if key == "tiny-deepseek-v4":
        from .deepseek_v4.config import DeepseekV4Config

        return DeepseekV4Config(**{**TINY_DEEPSEEK_V4, **(overrides or {})})
    if key in GENERIC_PRESETS:
        from .hf_generic import HFGenericConfig

        return HFGenericConfig({**GENERIC_PRESETS[key], **(overrides or {})})
    if key in PRESETS:
        cfg = PRESETS[key]
    else:
        p = Path(name)
        if p.is_dir() and (p / "config.json").exists():
            p = p / "config.json"
        if p.is_file():
            d = json.loads(p.read_text())
            if d.get("model_type") == "deepseek_v4":
                from .deepseek_v4.config import DeepseekV4Config

                cfg = DeepseekV4Config.from_dict(d)
                return DeepseekV4Config.from_dict({**cfg.to_dict(), **(overrides or {})}) if overrides else cfg
            if d.get("model_type", "qwen3") not in ("qwen2", "qwen3", "qwen3_moe") and "model_type" in d:
                from .hf_generic import HFGenericConfig

                return HFGenericConfig({**d, **(overrides or {})}, source=str(p.parent))
            cfg = from_hf_config(d)
        else:
            raise ValueError(
                f"unknown model {name!r}: not a preset ({', '.join(sorted(PRESETS))}), "
                "alias, or local Hugging Face directory"
            )
    if overrides:
        cfg = replace(cfg, **overrides)
    return cfg
