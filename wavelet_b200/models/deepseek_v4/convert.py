"""Published DeepSeek-V4 checkpoints <-> native tensors (reference
trainer/models/deepseek_v4/conversion.py, dequantize.py).

The published ("raw") layout names tensors ``layers.{i}.attn.wq_a.weight``,
``layers.{i}.ffn.experts.{e}.w1.weight`` and so on, stores routed experts one
tensor per expert, and may quantize weights: FP8 e4m3 or MXFP4 (two e2m1
codes per int8 byte, low nibble first) with a ``.scale`` tensor per block
grid.  Import dequantizes (to bf16) and stacks experts into [E, ...]
tensors; export writes plain tensors under the raw names.  ``mtp.*``
(multi-token prediction) tensors are skipped on import.

``python -m wavelet_b200.models.deepseek_v4.convert SRC DST [--to-raw]``
"""

from __future__ import annotations

import json
import re
from collections import defaultdict
from pathlib import Path

import torch
from torch import Tensor

# e2m1 code -> value (sign bit 3, exponent bits 2..1, mantissa bit 0)
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])

# (raw suffix, native suffix) inside one layer
LAYER_NAMES = [
    ("attn_norm.weight", "input_layernorm.weight"), ("ffn_norm.weight", "post_attention_layernorm.weight"),
    ("hc_attn_fn", "attn_hc.fn"), ("hc_attn_base", "attn_hc.base"), ("hc_attn_scale", "attn_hc.scale"),
    ("hc_ffn_fn", "ffn_hc.fn"), ("hc_ffn_base", "ffn_hc.base"), ("hc_ffn_scale", "ffn_hc.scale"),
    ("attn.wq_a.weight", "self_attn.q_a_proj.weight"), ("attn.q_norm.weight", "self_attn.q_a_norm.weight"),
    ("attn.wq_b.weight", "self_attn.q_b_proj.weight"), ("attn.wkv.weight", "self_attn.kv_proj.weight"),
    ("attn.kv_norm.weight", "self_attn.kv_norm.weight"), ("attn.wo_a.weight", "self_attn.o_a_proj.weight"),
    ("attn.wo_b.weight", "self_attn.o_b_proj.weight"), ("attn.attn_sink", "self_attn.sinks"),
    ("ffn.gate.weight", "mlp.router.gate.weight"), ("ffn.gate.bias", "mlp.router.selection_bias"),
    ("ffn.gate.tid2eid", "mlp.router.tid2eid"),
    ("ffn.shared_experts.w1.weight", "mlp.shared_expert.gate_proj.weight"),
    ("ffn.shared_experts.w2.weight", "mlp.shared_expert.down_proj.weight"),
    ("ffn.shared_experts.w3.weight", "mlp.shared_expert.up_proj.weight"),
]
COMPRESSOR_NAMES = [("wkv.weight", "kv_proj.weight"), ("wgate.weight", "gate_proj.weight"),
                    ("norm.weight", "kv_norm.weight"), ("ape", "position_bias")]
INDEXER_NAMES = [("wq_b.weight", "q_b_proj.weight"), ("weights_proj.weight", "weights_proj.weight")]
GLOBAL_NAMES = {"embed.weight": "model.embed_tokens.weight", "head.weight": "lm_head.weight",
                "norm.weight": "model.norm.weight", "hc_head_fn": "model.hc_head.hc_fn",
                "hc_head_base": "model.hc_head.hc_base", "hc_head_scale": "model.hc_head.hc_scale"}
EXPERT_W = {"w1": "gate_proj", "w2": "down_proj", "w3": "up_proj"}
RAW_EXPERT = re.compile(r"^layers\.(\d+)\.ffn\.experts\.(\d+)\.(w[123])\.weight$")
NATIVE_EXPERT = re.compile(r"^model\.layers\.(\d+)\.mlp\.experts\.(gate_proj|up_proj|down_proj)$")


def _name_table(layer_ids) -> dict[str, str]:
    """raw name -> native name for every tensor a layer may own (the
    compressor / indexer entries only match in layers that have them)."""
    table = dict(GLOBAL_NAMES)
    for i in layer_ids:
        r, n = f"layers.{i}.", f"model.layers.{i}."
        table.update({r + a: n + b for a, b in LAYER_NAMES})
        table.update({f"{r}attn.compressor.{a}": f"{n}self_attn.compressor.{b}" for a, b in COMPRESSOR_NAMES})
        table.update({f"{r}attn.indexer.{a}": f"{n}self_attn.compressor.indexer.{b}" for a, b in INDEXER_NAMES})
        table.update({f"{r}attn.indexer.compressor.{a}": f"{n}self_attn.compressor.indexer.compressor.{b}"
                      for a, b in COMPRESSOR_NAMES})
    return table


def _layers_of(keys) -> set[int]:
    out = set()
    for k in keys:
        m = re.match(r"^(?:model\.)?layers\.(\d+)\.", k)
        if m:
            out.add(int(m.group(1)))
    return out


# ----------------------------------------------------------- dequantization
def unpack_mxfp4(packed: Tensor) -> Tensor:
    b = packed.contiguous().view(torch.uint8)
    lut = E2M1.to(packed.device)
    lo, hi = lut[(b & 0xF).long()], lut[(b >> 4).long()]
    return torch.stack([lo, hi], dim=-1).flatten(-2)


def dequantize(weight: Tensor, scale: Tensor) -> Tensor:
    if weight.dtype == torch.int8:
        v = unpack_mxfp4(weight)
    elif weight.dtype == torch.float8_e4m3fn:
        v = weight.float()
    else:
        raise ValueError(f"unsupported quantized weight dtype {weight.dtype}")
    R, C = v.shape[-2:]
    sr, sc = scale.shape[-2:]
    if R % sr or C % sc:
        raise ValueError(f"weight {tuple(v.shape[-2:])} is not a multiple of its scale grid {tuple(scale.shape[-2:])}")
    s = scale.float().repeat_interleave(R // sr, -2).repeat_interleave(C // sc, -1)
    return (v * s).to(torch.bfloat16)


def dequantize_state_(state: dict[str, Tensor]) -> None:
    for key in [k for k in state if k.endswith(".weight")]:
        skey = key[: -len(".weight")] + ".scale"
        quantized = state[key].dtype in (torch.int8, torch.float8_e4m3fn)
        if quantized and skey not in state:
            raise ValueError(f"quantized weight {key} has no scale tensor")
        if skey in state:
            state[key] = dequantize(state[key], state.pop(skey))


# --------------------------------------------------------------- mapping
def raw_to_native(raw: dict[str, Tensor]) -> dict[str, Tensor]:
    state = dict(raw)
    dequantize_state_(state)
    table = _name_table(_layers_of(state))
    out: dict[str, Tensor] = {}
    experts: dict[tuple[int, str], dict[int, Tensor]] = defaultdict(dict)
    for k, v in state.items():
        if k.startswith("mtp."):
            continue
        m = RAW_EXPERT.match(k)
        if m:
            experts[int(m.group(1)), EXPERT_W[m.group(3)]][int(m.group(2))] = v
        elif k in table:
            out[table[k]] = v
        else:
            raise ValueError(f"unrecognised DeepSeek-V4 raw checkpoint tensor {k}")
    for (layer, proj), by_id in experts.items():
        if sorted(by_id) != list(range(len(by_id))):
            raise ValueError("DeepSeek-V4 expert ids must run 0..E-1 without gaps")
        out[f"model.layers.{layer}.mlp.experts.{proj}"] = torch.stack([by_id[e] for e in range(len(by_id))])
    return out


def native_to_raw(native: dict[str, Tensor]) -> dict[str, Tensor]:
    inverse = {v: k for k, v in _name_table(_layers_of(native)).items()}
    w_of = {v: k for k, v in EXPERT_W.items()}
    out: dict[str, Tensor] = {}
    for k, v in native.items():
        m = NATIVE_EXPERT.match(k)
        if m:
            if v.dim() != 3:
                raise ValueError("DeepSeek-V4 stacked expert weights must be 3-D")
            for e, t in enumerate(v.unbind(0)):
                out[f"layers.{m.group(1)}.ffn.experts.{e}.{w_of[m.group(2)]}.weight"] = t
        elif k in inverse:
            out[inverse[k]] = v
        else:
            raise ValueError(f"unrecognised DeepSeek-V4 native tensor {k}")
    return out


def _load_dir(src: Path) -> dict[str, Tensor]:
    from safetensors.torch import load_file

    index = src / "model.safetensors.index.json"
    files = sorted(set(json.loads(index.read_text())["weight_map"].values())) if index.exists() else [
        "model.safetensors"]
    state: dict[str, Tensor] = {}
    for f in files:
        path = src / f
        if path.resolve().parent != src.resolve():
            raise ValueError("checkpoint shards must sit directly in the source folder")
        shard = load_file(str(path), device="cpu")
        dup = state.keys() & shard.keys()
        if dup:
            raise ValueError(f"duplicate checkpoint tensors: {sorted(dup)}")
        state.update(shard)
    return state


def convert_checkpoint(src: str | Path, dst: str | Path, to_raw: bool = False) -> None:
    """Convert a local safetensors checkpoint (all weights in CPU memory).
    The destination must not exist; it is only created once the converted
    tensors match the model's names and shapes."""
    from safetensors.torch import save_file

    from .config import CHECKPOINT_FORMAT, DeepseekV4Config
    from .model import DeepseekV4ForCausalLM

    src, dst = Path(src), Path(dst)
    if dst.exists():
        raise FileExistsError(f"checkpoint destination exists: {dst}")
    cfg = DeepseekV4Config.from_pretrained(src)
    state = _load_dir(src)
    converted = native_to_raw(state) if to_raw else raw_to_native(state)
    if not converted:
        raise ValueError("the checkpoint holds no model weights")
    native = state if to_raw else converted
    with torch.device("meta"):
        expected = DeepseekV4ForCausalLM(cfg, init=False).state_dict()
    missing = sorted(expected.keys() - native.keys())
    extra = sorted(native.keys() - expected.keys())
    shapes = sorted(k for k in expected.keys() & native.keys() if tuple(expected[k].shape) != tuple(native[k].shape))
    if missing or extra or shapes:
        raise ValueError(f"invalid DeepSeek-V4 checkpoint: missing={missing}, unexpected={extra}, wrong shape={shapes}")
    dst.mkdir(parents=True)
    save_file({k: v.contiguous() for k, v in converted.items()}, str(dst / "model.safetensors"))
    cfg.set_extra("wavelet_checkpoint_format", None if to_raw else CHECKPOINT_FORMAT)
    cfg.set_extra("quantization_config", None)
    cfg.set_extra("architectures", ["DeepseekV4ForCausalLM"])
    cfg.save_pretrained(dst)


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="Convert local DeepSeek-V4 safetensors checkpoints.")
    ap.add_argument("source", type=Path)
    ap.add_argument("target", type=Path)
    ap.add_argument("--to-raw", action="store_true")
    a = ap.parse_args(argv)
    convert_checkpoint(a.source, a.target, to_raw=a.to_raw)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
