"""``wavelet convert-checkpoint``: a stable ``checkpoint-N`` directory to
Hugging Face safetensors (reference tools/convert_checkpoint.py).

Full fine-tune checkpoints hold the internal flat tensor names in
``trainer/model.safetensors``; they are mapped to HF names and re-sharded.
LoRA checkpoints hold adapter tensors (``l<i>.<target>.A/B``); they are
written as a PEFT adapter (``adapter_model.safetensors`` +
``adapter_config.json``).  The model architecture comes from ``meta.json``
(saved by the trainer) or from ``--config``.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _parse_size(s: str) -> int:
    s = s.strip().upper()
    for unit, mul in (("GB", 1 << 30), ("MB", 1 << 20), ("KB", 1 << 10), ("B", 1)):
        if s.endswith(unit):
            return int(float(s[: -len(unit)]) * mul)
    return int(s)


def convert_checkpoint(ckpt: Path, output_dir: Path | None = None, config_path: Path | None = None,
                       dtype: str = "bfloat16", max_shard_size: str = "5GB") -> Path:
    from safetensors.torch import load_file

    from ..models.config import ArchConfig, resolve_arch
    from ..models.qwen import build_model

    ckpt = Path(ckpt)
    root = ckpt.parent if ckpt.name == "trainer" else ckpt
    if not (root / "STABLE").exists():
        raise FileNotFoundError(f"{root} is not a stable checkpoint (no STABLE marker)")
    meta = json.loads((root / "meta.json").read_text())
    out = Path(output_dir) if output_dir else root / "weights"
    if meta.get("arch", {}).get("model_type") == "deepseek_v4":
        return _convert_deepseek_v4(root, meta, out, DTYPES[dtype])
    if "arch" in meta:
        arch = ArchConfig.from_dict(meta["arch"]) if hasattr(ArchConfig, "from_dict") else ArchConfig(**meta["arch"])
    elif config_path is not None:
        from ..utils.config import load_yaml

        arch = resolve_arch(load_yaml(config_path)["model"]["name"])
    else:
        raise ValueError("checkpoint has no architecture metadata; pass --config")
    tensors = load_file(str(root / "trainer" / "model.safetensors"))
    lora_keys = [k for k in tensors if k.endswith(".A") or k.endswith(".B")]
    if lora_keys:
        from types import SimpleNamespace

        from ..models.lora import LoRAAdapters

        rank = meta.get("lora_rank")
        targets = meta.get("lora_target_modules")
        alpha = meta.get("lora_alpha")
        if rank is None or targets is None or alpha is None:
            raise ValueError("LoRA checkpoint meta.json lacks lora_rank / lora_alpha / lora_target_modules")
        ad = LoRAAdapters(arch, int(rank), float(alpha), list(targets), "cpu", torch.float32)
        ad.flat.load_state({k: v.float() for k, v in tensors.items()})
        ad.save_adapter(out, base_model=meta.get("model_name"))
        return out
    model = build_model(arch, "cpu", DTYPES[dtype], init=False, with_grad=False, with_optimizer=False)
    model.flat.load_state({k: v.to(DTYPES[dtype]) for k, v in tensors.items()})
    from ..models.hf_io import save_hf

    save_hf(model, out, dtype=DTYPES[dtype], max_shard_bytes=_parse_size(max_shard_size))
    return out


def _convert_deepseek_v4(root: Path, meta: dict, out: Path, dtype: torch.dtype) -> Path:
    """DeepSeek-V4 checkpoints hold native tensor names in two stores (the
    compute-dtype store and the fp32 store of the sensitive tensors); the
    output is a native checkpoint directory (config.json + model.safetensors)
    that ``DeepseekV4ForCausalLM.from_pretrained`` loads and
    ``models.deepseek_v4.convert`` turns into the published layout."""
    from safetensors.torch import load_file

    from ..models.deepseek_v4 import DeepseekV4Config, DeepseekV4ForCausalLM

    cfg = DeepseekV4Config.from_dict(meta["arch"])
    state = load_file(str(root / "trainer" / "model.safetensors"))
    for extra in ("experts-ep0.safetensors", "extra.safetensors"):  # fp32 store; routing buffers
        if (root / "trainer" / extra).exists():
            state.update(load_file(str(root / "trainer" / extra)))
    model = DeepseekV4ForCausalLM(cfg, init=False)
    missing = set(dict(model.named_parameters())) - set(state)
    if missing:
        raise ValueError(f"DeepSeek-V4 checkpoint lacks {sorted(missing)[:5]} ...")
    with torch.no_grad():
        params, buffers = dict(model.named_parameters()), dict(model.named_buffers())
        for k, v in state.items():
            if k in params:
                params[k].copy_(v.float())
            elif k in buffers:
                buffers[k].copy_(v.to(buffers[k].dtype))
    model.to_compute_dtype(dtype)
    model.save_pretrained(out)
    return out


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="wavelet convert-checkpoint", description=__doc__)
    p.add_argument("checkpoint", type=Path, help="stable checkpoint-N directory or its trainer subdirectory")
    p.add_argument("output_dir", type=Path, nargs="?", help="destination (default: <checkpoint>/weights)")
    p.add_argument("--config", type=Path, help="run config when the checkpoint has no architecture metadata")
    p.add_argument("--dtype", choices=tuple(DTYPES), default="bfloat16")
    p.add_argument("--max-shard-size", default="5GB")
    a = p.parse_args(sys.argv[1:] if argv is None else argv)
    out = convert_checkpoint(a.checkpoint, a.output_dir, a.config, a.dtype, a.max_shard_size)
    print(f"Converted checkpoint to {out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
