"""Model-section options that act after the model is built.

* ``model.matmul_precision`` -> ``torch.set_float32_matmul_precision`` (the
  float32 torch matmuls: CPU paths, Muon's Newton-Schulz, the eager
  DeepSeek-V4 model), as the reference does at set-up.
* ``model.moe_router_dtype``: ``none`` keeps the router gate in the model
  dtype (bf16 logits, as a bf16 ``nn.Linear`` gate produces); ``float32``
  keeps the fp32 logits of the router GEMM (reference trainer/moe.py:298).
* ``model.freeze_moe_router``: the router weights are frozen (no gradient,
  no update, no decay); a model without MoE routers is an error, as in the
  reference (trainer/moe.py:275-300).
* ``model.meta_device_init`` asks the reference's FSDP wrapper to build on
  the meta device: here parameters are always allocated directly on the
  device (each rank only its shard with ``fsdp.shard_params``), so it is
  satisfied as it is; setting it logs that.
* ``fsdp.reshard_after_forward``: with ``fsdp.shard_params`` (ZeRO-3) the
  gathered weights of a layer are released after its forward and gathered
  again for its backward, which is the reference's ``true``; without
  sharded parameters the bf16 weights stay resident on every rank.
"""

from __future__ import annotations

import logging

import torch

log = logging.getLogger("wavelet")


def lm_head_chunk(mcfg) -> int:
    """Tokens per LM-head chunk: ``model.fused_lm_head_token_chunk_size``
    when it is a number; the loss is always chunked, so ``auto`` and
    ``disabled`` (the reference's unfused head) use the default chunk."""
    from ..ops.lm_head import DEFAULT_CHUNK

    v = getattr(mcfg, "fused_lm_head_token_chunk_size", None)
    return int(v) if isinstance(v, int) and not isinstance(v, bool) and v > 0 else DEFAULT_CHUNK


def apply_model_options(model, mcfg, fsdp_cfg=None, trainer_cfg=None) -> list[str]:
    notes: list[str] = []
    prec = getattr(mcfg, "matmul_precision", None)
    if prec:
        torch.set_float32_matmul_precision(prec)
    layers = getattr(model, "layers", [])
    routers = [layer.moe for layer in layers if getattr(layer, "moe", None) is not None]
    for moe in routers:
        moe.router_logits_bf16 = getattr(mcfg, "moe_router_dtype", "none") == "none"
    if getattr(mcfg, "freeze_moe_router", False):
        names = [n for n in model.flat.names() if n.endswith(".router_w")]
        if not routers or not names:
            raise ValueError("model.freeze_moe_router=true requires a model with MoE routers (a Qwen3-MoE shape)")
        model.freeze(names)
        notes.append(f"model.freeze_moe_router: {len(names)} router weights frozen")
    if trainer_cfg is not None and getattr(trainer_cfg, "activation_offloading", None) is not None \
            and hasattr(model, "enable_activation_offload"):
        model.enable_activation_offload()  # layer inputs kept in pinned host memory until the backward
        notes.append("activation_offloading: layer inputs offloaded to host memory")
    vlm = getattr(mcfg, "vlm", None)
    if vlm is not None and getattr(vlm, "freeze_vision_encoder", False) and hasattr(model, "freeze_prefix"):
        n = model.freeze_prefix(vlm.vision_encoder_attr)
        notes.append(f"model.vlm.freeze_vision_encoder: {n} vision-tower parameters frozen")
    if getattr(mcfg, "meta_device_init", False):
        notes.append("model.meta_device_init: parameters are allocated directly on the device "
                     "(no host materialisation to defer)")
    if fsdp_cfg is not None and "reshard_after_forward" in getattr(fsdp_cfg, "model_fields_set", set()):
        if getattr(fsdp_cfg, "shard_params", False):
            notes.append("fsdp.reshard_after_forward: sharded parameters are gathered per layer, released after "
                         "the forward and gathered again in the backward")
        else:
            notes.append(f"fsdp.reshard_after_forward={fsdp_cfg.reshard_after_forward}: bf16 weights stay "
                         "resident on every data-parallel rank (only optimizer state is sharded; "
                         "fsdp.shard_params shards them)")
    for n in notes:
        log.info(n)
    return notes
