"""Settings that the reference's schema has and that do nothing here.

The configuration schema keeps the reference's keys so its YAML files load
unchanged, but some of them configure machinery this framework replaced
(vLLM's engine, PEFT, ``torch.compile``, Liger kernels, DataLoader workers).
A user who sets one of them must not get a silently different run:
``inert_settings`` lists every such key the config sets away from its default,
with the reason, and the trainers and the rollout role log them at start-up
(``warn_inert``).  Keys whose effect this framework implements differently
(for example ``inference.vllm.enforce_eager``, which turns off the native
generator's CUDA graphs) are not listed here.
"""

from __future__ import annotations

import logging
from typing import Any

log = logging.getLogger("wavelet")

_GENERATOR = "the native generator has no such setting"

INERT: dict[str, str] = {
    "model.experts_implementation": "MoE experts always run as grouped tcgen05 GEMMs",
    "model.kbit_cast_non_quantized_to_float32": "non-quantised QLoRA parameters stay in the flat store's dtype "
                                                "with fp32 master copies",
    "model.fused_lora_mlp": "LoRA is always fused into the projection GEMMs",
    "model.fused_lora_qkv": "LoRA is always fused into the projection GEMMs",
    "model.fused_lora_o": "LoRA is always fused into the projection GEMMs",
    "model.compile": "layers run fixed sm_100a kernel sequences; torch.compile is not used",
    "model.compile_fullgraph": "layers run fixed sm_100a kernel sequences; torch.compile is not used",
    "lora.optimization_dtype": "LoRA adapters always keep fp32 master weights and moments",
    "optim.implementation": "AdamW is the fused flat kernel",
    "data.num_workers": "rollout rows are pretokenized and read in the trainer process",
    "loss_impl": "the loss is the chunked LM-head kernel",
    "slurm.shared_fs": "role configs and logs are written under the run directory in every case",
    "policy_transfer.nccl_dtype": "device updates carry the generator's compute dtype",
    "inference.vllm.quantization": _GENERATOR,
    "inference.vllm.load_format": _GENERATOR,
    "inference.vllm.data_parallel_size": "generator replicas are launcher.inference_num_replicas",
    "inference.vllm.data_parallel_size_local": _GENERATOR,
    "inference.vllm.data_parallel_rpc_port": _GENERATOR,
    "inference.vllm.fully_sharded_loras": _GENERATOR,
    "inference.vllm.enable_fp32_lm_head": "the generator samples from bf16 logits of an fp32-accumulated GEMM",
    "inference.vllm.enable_fp32_router_logits": "router logits follow model.moe_router_dtype",
    "inference.vllm.use_generation_logprobs": "generation log-probs always come from the sampling kernel",
    "inference.vllm.extra_args": "there is no vLLM engine to pass them to",
    "inference.sampling.extra_body": "the native sampler has no extra request fields (verifiers-package "
                                     "rollouts pass them to the server)",
    "orchestrator.max_pending_rollout_chunks": "in-flight steps are bounded by max_async_level",
    "data.pack_sequences": "RL rows are always packed as variable-length sequences that never attend across each "
                           "other, which trains the same loss as unpacked rows",
    "data.pad_to_multiple_of": "packed rows are variable-length; the kernels need no padding",
    "model.attn_implementation": "attention is the native variable-length tcgen05 kernel",
    "fsdp.impl": "parameters are sharded by the flat ZeRO store (fsdp.shard_params), not torch FSDP",
}


# keys that take effect in SFT and are inert only in RL configs
RL_ONLY = frozenset({"data.num_workers"})


def _lookup(cfg: Any, path: str) -> tuple[Any, str] | None:
    obj = cfg
    parts = path.split(".")
    for p in parts[:-1]:
        obj = getattr(obj, p, None)
        if obj is None:
            return None
    if not hasattr(obj, "model_fields_set") or parts[-1] not in type(obj).model_fields:
        return None
    return obj, parts[-1]


def inert_settings(cfg: Any) -> list[str]:
    """One message per inert key that ``cfg`` sets to a non-default value."""
    out = []
    rl = hasattr(cfg, "orchestrator")
    for path, why in INERT.items():
        if path in RL_ONLY and not rl:
            continue  # acts in SFT (data.num_workers: batches prefetched on a thread)
        hit = _lookup(cfg, path)
        if hit is None:
            continue
        obj, name = hit
        if name not in obj.model_fields_set:
            continue
        field = type(obj).model_fields[name]
        default = field.get_default(call_default_factory=True)
        if getattr(obj, name) == default:
            continue
        out.append(f"{path}={getattr(obj, name)!r} has no effect here: {why}")
    return out


def warn_inert(cfg: Any) -> list[str]:
    msgs = inert_settings(cfg)
    for m in msgs:
        log.warning(m)
    return msgs
