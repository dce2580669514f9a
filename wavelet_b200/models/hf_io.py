"""Hugging Face checkpoint interop (safetensors).

Internal fused tensors map to HF names:

    embed                 model.embed_tokens.weight
    l{i}.in_norm          model.layers.{i}.input_layernorm.weight
    l{i}.qkv_w            q_proj / k_proj / v_proj .weight  (row blocks)
    l{i}.qkv_b            q_proj / k_proj / v_proj .bias    (Qwen2)
    l{i}.q_norm, k_norm   self_attn.q_norm / k_norm .weight (Qwen3)
    l{i}.o_w              self_attn.o_proj.weight
    l{i}.post_norm        post_attention_layernorm.weight
    l{i}.gu_w             mlp.gate_proj / up_proj .weight   (row blocks)
    l{i}.down_w           mlp.down_proj.weight
    l{i}.router_w         mlp.gate.weight                   (Qwen3-MoE)
    l{i}.exp_gu_w[e]      mlp.experts.{e}.gate_proj / up_proj .weight
    l{i}.exp_down_w[e]    mlp.experts.{e}.down_proj.weight
    norm                  model.norm.weight
    lm_head               lm_head.weight                    (untied)

Used by model loading (trainer/model.py:536 / :837 in the reference), the
final HF export (:1273-1314) and ``convert-checkpoint``.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch


def hf_state_dict(model) -> dict[str, torch.Tensor]:
    if hasattr(model, "hf_state_dict"):  # a transformers module: its own names
        return model.hf_state_dict()
    cfg = model.cfg
    f = model.flat
    q, kv = cfg.q_dim, cfg.kv_dim
    out: dict[str, torch.Tensor] = {"model.embed_tokens.weight": f.view("embed")}
    for i in range(cfg.num_layers):
        p, h = f"l{i}.", f"model.layers.{i}."
        out[h + "input_layernorm.weight"] = f.view(p + "in_norm")
        w = f.view(p + "qkv_w")
        out[h + "self_attn.q_proj.weight"] = w[:q]
        out[h + "self_attn.k_proj.weight"] = w[q : q + kv]
        out[h + "self_attn.v_proj.weight"] = w[q + kv :]
        if cfg.qkv_bias:
            b = f.view(p + "qkv_b")
            out[h + "self_attn.q_proj.bias"] = b[:q]
            out[h + "self_attn.k_proj.bias"] = b[q : q + kv]
            out[h + "self_attn.v_proj.bias"] = b[q + kv :]
        if cfg.qk_norm:
            out[h + "self_attn.q_norm.weight"] = f.view(p + "q_norm")
            out[h + "self_attn.k_norm.weight"] = f.view(p + "k_norm")
        out[h + "self_attn.o_proj.weight"] = f.view(p + "o_w")
        out[h + "post_attention_layernorm.weight"] = f.view(p + "post_norm")
        if cfg.layer_is_moe(i):
            out[h + "mlp.gate.weight"] = f.view(p + "router_w")
            gu = f.view(p + "exp_gu_w")
            dn = f.view(p + "exp_down_w")
            Ie = cfg.moe_intermediate_size
            for e in range(cfg.num_experts):
                out[h + f"mlp.experts.{e}.gate_proj.weight"] = gu[e, :Ie]
                out[h + f"mlp.experts.{e}.up_proj.weight"] = gu[e, Ie:]
                out[h + f"mlp.experts.{e}.down_proj.weight"] = dn[e]
        else:
            I = cfg.intermediate_size
            gu = f.view(p + "gu_w")
            out[h + "mlp.gate_proj.weight"] = gu[:I]
            out[h + "mlp.up_proj.weight"] = gu[I:]
            out[h + "mlp.down_proj.weight"] = f.view(p + "down_w")
    out["model.norm.weight"] = f.view("norm")
    if not cfg.tie_embeddings:
        out["lm_head.weight"] = f.view("lm_head")
    return out


def internal_from_hf(cfg, hf: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Inverse mapping: HF tensors -> internal fused tensors."""
    t: dict[str, torch.Tensor] = {"embed": hf["model.embed_tokens.weight"], "norm": hf["model.norm.weight"]}
    for i in range(cfg.num_layers):
        p, h = f"l{i}.", f"model.layers.{i}."
        t[p + "in_norm"] = hf[h + "input_layernorm.weight"]
        t[p + "qkv_w"] = torch.cat([hf[h + f"self_attn.{x}_proj.weight"] for x in "qkv"], 0)
        if cfg.qkv_bias:
            t[p + "qkv_b"] = torch.cat([hf[h + f"self_attn.{x}_proj.bias"] for x in "qkv"], 0)
        if cfg.qk_norm:
            t[p + "q_norm"] = hf[h + "self_attn.q_norm.weight"]
            t[p + "k_norm"] = hf[h + "self_attn.k_norm.weight"]
        t[p + "o_w"] = hf[h + "self_attn.o_proj.weight"]
        t[p + "post_norm"] = hf[h + "post_attention_layernorm.weight"]
        if cfg.layer_is_moe(i):
            t[p + "router_w"] = hf[h + "mlp.gate.weight"]
            t[p + "exp_gu_w"] = torch.stack([torch.cat([hf[h + f"mlp.experts.{e}.gate_proj.weight"], hf[h + f"mlp.experts.{e}.up_proj.weight"]], 0) for e in range(cfg.num_experts)])
            t[p + "exp_down_w"] = torch.stack([hf[h + f"mlp.experts.{e}.down_proj.weight"] for e in range(cfg.num_experts)])
        else:
            t[p + "gu_w"] = torch.cat([hf[h + "mlp.gate_proj.weight"], hf[h + "mlp.up_proj.weight"]], 0)
            t[p + "down_w"] = hf[h + "mlp.down_proj.weight"]
    if not cfg.tie_embeddings:
        t["lm_head"] = hf.get("lm_head.weight", hf["model.embed_tokens.weight"])
    return t


def load_hf_weights(model, path: Path) -> None:
    from safetensors.torch import load_file

    if getattr(model.cfg, "generic_hf", False):  # a transformers module: its own checkpoint names
        model.load_pretrained(path)
        return
    if hasattr(model, "load_pretrained"):  # eager DeepSeek-V4: native checkpoint directory
        cfg_file = Path(path) / "config.json"
        if cfg_file.exists() and json.loads(cfg_file.read_text()).get("wavelet_checkpoint_format") is None:
            raise ValueError(f"{path} is a published DeepSeek-V4 checkpoint; convert it to a converted native "
                             "checkpoint first (python -m wavelet_b200.models.deepseek_v4.convert)")
        model.load_pretrained(path)
        return

    files = sorted(Path(path).glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    hf: dict[str, torch.Tensor] = {}
    for fp in files:
        hf.update(load_file(str(fp)))
    tensors = internal_from_hf(model.cfg, hf)
    tp = getattr(model, "tp_size", 1)
    if tp > 1:  # this rank's Megatron part of every split parameter
        from .qwen import tp_slicers

        sl = tp_slicers(model.cfg, tp, model.tp_rank)
        tensors = {n: (sl[n.split(".", 1)[-1]][1](t) if n.split(".", 1)[-1] in sl else t) for n, t in tensors.items()}
    model.flat.load_state(tensors)
    ef = getattr(model, "expert_flat", None)
    if ef is not None:  # expert parallelism: this rank's block of experts
        el = model.cfg.num_experts // model.ep_size
        lo = model.ep_rank * el
        ef.load_state({n: tensors[n][lo:lo + el] for n in ef.names()})
    if getattr(model, "quant", None):
        from ..ops.nf4 import quantize

        for name, q in model.quant.items():  # QLoRA: quantise the loaded projections in place
            nq = quantize(tensors[name].to(device=q.device, dtype=model.flat.compute_dtype))
            q.codes.copy_(nq.codes)
            q.absmax.copy_(nq.absmax)
            q.version += 1


def save_hf(model, out_dir: Path, dtype: torch.dtype = torch.bfloat16, max_shard_bytes: int = 5 * 2**30) -> list[Path]:
    """Write HF-layout safetensors shards + config.json (+ index for >1 shard)."""
    from safetensors.torch import save_file

    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    sd = {k: v.detach().to("cpu", dtype).contiguous() for k, v in hf_state_dict(model).items()}
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for k, v in sd.items():
        nb = v.numel() * v.element_size()
        if size + nb > max_shard_bytes and shards[-1]:
            shards.append({})
            size = 0
        shards[-1][k] = v
        size += nb
    paths = []
    index = {}
    for i, sh in enumerate(shards):
        name = "model.safetensors" if len(shards) == 1 else f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, str(out_dir / name), metadata={"format": "pt"})
        paths.append(out_dir / name)
        for k in sh:
            index[k] = name
    if len(shards) > 1:
        (out_dir / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": index}, indent=2))
    cfgd = model.cfg.to_hf_config()
    cfgd["torch_dtype"] = str(dtype).replace("torch.", "")
    (out_dir / "config.json").write_text(json.dumps(cfgd, indent=2))
    return paths
