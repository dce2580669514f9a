"""LoRA adapters on the fused linear layers of a decoder.

PEFT semantics (the reference wraps its HF model with ``peft.get_peft_model``,
trainer/model.py:1512-1545, and runs the adapters through its fused autograd
kernels, kernels/lora.py:59-291):

    y = x W^T + (alpha / r) * (x A^T) B^T,   A: [r, in] (Kaiming-uniform init),
                                            B: [out, r] (zero init)

Our decoder keeps q/k/v as one fused ``qkv_w`` and gate/up as one ``gu_w``, so
the adapters of a fused linear are stacked: ``A`` [kp, in] holds the A
matrices of its enabled parts (q, k, v or gate, up) in r-row slots and ``B``
[out, kp] holds each part's B in its own row block and slot columns (a
block-diagonal layout).  kp is the slot total rounded up to 64 so the adapter
product is whole k-blocks of the tcgen05 GEMM.  Off-diagonal blocks and padding
stay exactly zero: their gradients are never applied.

GPU linear with an adapter (csrc/gemm.cu, second operand pair):

    forward   u  = s x A^T            (thin GEMM, alpha = s)
              y  = x W^T + u B^T      (ONE GEMM: base k-blocks then kp/64 adapter k-blocks)
    backward  dB = dy^T u             (block-diagonal part only)
              g  = s dy B             (thin GEMM)
              dA += g^T x
              dx = dy W + g A         (ONE GEMM, B operands MN-major)

The adapters live in their own ``FlatParams`` store, so the optimizer, the
gradient reduce-scatter and checkpoints see only the trainable parameters;
the base model's store is frozen (no gradient buffer at all).
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass
from pathlib import Path

import torch

from .config import ArchConfig
from .params import FlatParams, ParamSpec

SLOT_ALIGN = 64

# fused linear -> (weight name, [(peft module, attribute path)])
_TARGETS = {
    "qkv": ("qkv_w", [("q_proj", "self_attn"), ("k_proj", "self_attn"), ("v_proj", "self_attn")]),
    "o": ("o_w", [("o_proj", "self_attn")]),
    "gu": ("gu_w", [("gate_proj", "mlp"), ("up_proj", "mlp")]),
    "down": ("down_w", [("down_proj", "mlp")]),
}


def _part_rows(cfg: ArchConfig, target: str) -> list[tuple[int, int]]:
    if target == "qkv":
        q, kv = cfg.q_dim, cfg.kv_dim
        return [(0, q), (q, q + kv), (q + kv, q + 2 * kv)]
    if target == "o":
        return [(0, cfg.hidden_size)]
    if target == "gu":
        i = cfg.intermediate_size
        return [(0, i), (i, 2 * i)]
    return [(0, cfg.hidden_size)]


def _in_dim(cfg: ArchConfig, target: str) -> int:
    return {"qkv": cfg.hidden_size, "o": cfg.q_dim, "gu": cfg.hidden_size, "down": cfg.intermediate_size}[target]


def _out_dim(cfg: ArchConfig, target: str) -> int:
    return _part_rows(cfg, target)[-1][1]


@dataclass
class TargetLayout:
    target: str
    weight: str
    in_dim: int
    out_dim: int
    kp: int
    # enabled parts: (peft module name, attr path, row lo, row hi, slot col lo)
    parts: list[tuple[str, str, int, int, int]]


@dataclass
class AdapterViews:
    """One fused linear's adapter in one layer (views into the flat stores)."""

    A: torch.Tensor  # [kp, in]
    B: torch.Tensor  # [out, kp]
    GA: torch.Tensor | None
    GB: torch.Tensor | None
    layout: TargetLayout
    scale: float
    rank: int

    @torch.no_grad()
    def add_b_grad(self, gB: torch.Tensor) -> None:
        """Accumulate the block-diagonal part of a full [out, kp] gradient."""
        if self.GB is None:
            return
        r = self.rank
        for _, _, lo, hi, c0 in self.layout.parts:
            self.GB[lo:hi, c0 : c0 + r] += gB[lo:hi, c0 : c0 + r].to(self.GB.dtype)


class LoRAAdapters:
    def __init__(self, cfg: ArchConfig, rank: int, alpha: float, target_modules: list[str], device,
                 dtype: torch.dtype, dp_rank: int = 0, dp_world: int = 1, dropout: float = 0.0,
                 seed: int = 0, fabric=None):
        if dropout > 0.0:
            raise ValueError("wavelet_b200 LoRA: lora.dropout must be 0 (the fused adapter kernels apply none)")
        self.cfg = cfg
        self.rank = rank
        self.alpha = alpha
        self.scale = alpha / rank
        self.target_modules = list(target_modules)
        wanted = set(target_modules)
        self.layouts: dict[str, TargetLayout] = {}
        for t, (wname, parts) in _TARGETS.items():
            rows = _part_rows(cfg, t)
            enabled = []
            for j, ((mod, path), (lo, hi)) in enumerate(zip(parts, rows)):
                if mod in wanted:
                    enabled.append((mod, path, lo, hi, len(enabled) * rank))
            if enabled:
                kp = (len(enabled) * rank + SLOT_ALIGN - 1) // SLOT_ALIGN * SLOT_ALIGN
                self.layouts[t] = TargetLayout(t, wname, _in_dim(cfg, t), _out_dim(cfg, t), kp, enabled)
        if not self.layouts:
            raise ValueError(f"no LoRA target among {sorted(wanted)} matches a dense projection of this model")
        self.moe_layers = [i for i in range(cfg.num_layers) if cfg.layer_is_moe(i)]
        specs: list[ParamSpec] = []
        for i in range(cfg.num_layers):
            for t, lay in self.layouts.items():
                if t in ("gu", "down") and cfg.layer_is_moe(i):
                    continue  # expert adapters are not supported; MoE layers keep dense attention adapters
                specs.append(ParamSpec(f"l{i}.{t}.A", (lay.kp, lay.in_dim), "zeros"))
                specs.append(ParamSpec(f"l{i}.{t}.B", (lay.out_dim, lay.kp), "zeros"))
        self.flat = FlatParams(specs, device, dtype, dp_rank, dp_world, True, True,
                               alloc=fabric.allocator() if fabric is not None else None)
        self.reset_parameters(seed)

    # ----------------------------------------------------------------- init
    @torch.no_grad()
    def reset_parameters(self, seed: int = 0) -> None:
        """A ~ U(-1/sqrt(in), 1/sqrt(in)) in the enabled slots (PEFT's Kaiming-uniform
        with a = sqrt(5)); B = 0; padding rows of A = 0."""
        g = torch.Generator(device=self.flat.device)
        for k, s in enumerate(self.flat.specs):
            v = self.flat.view(s.name)
            v.zero_()
            if s.name.endswith(".A"):
                t = s.name.split(".")[1]
                lay = self.layouts[t]
                bound = 1.0 / math.sqrt(lay.in_dim)
                g.manual_seed(seed * 1_000_003 + k)
                for _, _, _, _, c0 in lay.parts:
                    tmp = torch.empty(self.rank, lay.in_dim, device=self.flat.device, dtype=torch.float32)
                    tmp.uniform_(-bound, bound, generator=g)
                    v[c0 : c0 + self.rank].copy_(tmp)
        self.flat.sync_master_from_compute()

    # ---------------------------------------------------------------- views
    def layer_views(self, i: int) -> dict[str, AdapterViews]:
        out = {}
        for t, lay in self.layouts.items():
            a = f"l{i}.{t}.A"
            if a not in self.flat.offsets:
                continue
            b = f"l{i}.{t}.B"
            out[t] = AdapterViews(self.flat.view(a), self.flat.view(b), self.flat.grad_view(a),
                                  self.flat.grad_view(b), lay, self.scale, self.rank)
        return out

    def num_trainable(self) -> int:
        """Parameter count of the logical (unpadded) adapters."""
        n = 0
        for i in range(self.cfg.num_layers):
            for t, lay in self.layouts.items():
                if f"l{i}.{t}.A" in self.flat.offsets:
                    for _, _, lo, hi, _ in lay.parts:
                        n += self.rank * (lay.in_dim + (hi - lo))
        return n

    # ------------------------------------------------------------- PEFT I/O
    def peft_tensors(self) -> dict[str, torch.Tensor]:
        out = {}
        r = self.rank
        for i in range(self.cfg.num_layers):
            for t, lay in self.layouts.items():
                a = f"l{i}.{t}.A"
                if a not in self.flat.offsets:
                    continue
                A, B = self.flat.view(a), self.flat.view(f"l{i}.{t}.B")
                for mod, path, lo, hi, c0 in lay.parts:
                    pre = f"base_model.model.model.layers.{i}.{path}.{mod}"
                    out[pre + ".lora_A.weight"] = A[c0 : c0 + r].contiguous()
                    out[pre + ".lora_B.weight"] = B[lo:hi, c0 : c0 + r].contiguous()
        return out

    def save_adapter(self, path: Path, base_model: str | None = None) -> None:
        from safetensors.torch import save_file

        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        tensors = {k: v.detach().to("cpu") for k, v in self.peft_tensors().items()}
        save_file(tensors, str(path / "adapter_model.safetensors"))
        mods = sorted({m for lay in self.layouts.values() for m, *_ in lay.parts})
        (path / "adapter_config.json").write_text(json.dumps({
            "peft_type": "LORA", "task_type": "CAUSAL_LM", "r": self.rank, "lora_alpha": self.alpha,
            "lora_dropout": 0.0, "bias": "none", "target_modules": mods,
            "base_model_name_or_path": base_model,
        }, indent=2))

    @torch.no_grad()
    def load_peft_tensors(self, tensors: dict[str, torch.Tensor]) -> None:
        r = self.rank
        for i in range(self.cfg.num_layers):
            for t, lay in self.layouts.items():
                a = f"l{i}.{t}.A"
                if a not in self.flat.offsets:
                    continue
                A, B = self.flat.view(a), self.flat.view(f"l{i}.{t}.B")
                for mod, path, lo, hi, c0 in lay.parts:
                    pre = f"base_model.model.model.layers.{i}.{path}.{mod}"
                    A[c0 : c0 + r].copy_(tensors[pre + ".lora_A.weight"])
                    B[lo:hi, c0 : c0 + r].copy_(tensors[pre + ".lora_B.weight"])
        self.flat.sync_master_from_compute()

    # ---------------------------------------------------------------- merge
    @torch.no_grad()
    def merge_into(self, model) -> None:
        """W += s * B A for every adapted part of a dense bf16/fp32 model."""
        for i in range(self.cfg.num_layers):
            views = self.layer_views(i)
            for t, v in views.items():
                w = model.flat.view(f"l{i}.{v.layout.weight}")
                delta = (v.B.float() @ v.A.float()) * self.scale
                w.add_(delta.to(w.dtype))


def merge_adapter_into(model, adapter_dir: Path) -> None:
    """Merge a PEFT adapter directory into a dense model (generator policy load)."""
    from safetensors.torch import load_file

    adapter_dir = Path(adapter_dir)
    meta = json.loads((adapter_dir / "adapter_config.json").read_text())
    tensors = load_file(str(adapter_dir / "adapter_model.safetensors"))
    scale = float(meta["lora_alpha"]) / float(meta["r"])
    cfg = model.cfg
    with torch.no_grad():
        for t, (wname, parts) in _TARGETS.items():
            rows = _part_rows(cfg, t)
            for i in range(cfg.num_layers):
                name = f"l{i}.{wname}"
                if name not in model.flat.offsets:
                    continue
                w = model.flat.view(name)
                for (mod, path), (lo, hi) in zip(parts, rows):
                    pre = f"base_model.model.model.layers.{i}.{path}.{mod}"
                    if pre + ".lora_A.weight" not in tensors:
                        continue
                    A = tensors[pre + ".lora_A.weight"].to(w.device).float()
                    B = tensors[pre + ".lora_B.weight"].to(w.device).float()
                    w[lo:hi].add_((B @ A * scale).to(w.dtype))
