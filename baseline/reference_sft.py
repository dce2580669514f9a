"""Reference arm of ``bench.py``: the stock reference SFT trainer, timed.

This file drives the UNMODIFIED reference framework (a copy of its ``wavelet``
package in ``baseline/_ref``) through its own public Python API, the same
calls its ``wavelet sft`` command makes (``wavelet/trainer/trainer.py:1601-1690``):
``SFTConfig`` validation, ``validate_output_dir``, ``setup_config_logger``,
``SFTTrainer(config).setup()`` and ``SFTTrainer.train_until(step)``.  Nothing
of this repository's package is imported here, so its FSDP2 / NCCL / cuBLAS /
flash-attention path is what runs.

Two things are supplied from outside the reference tree because the box is
offline:

* ``baseline/shims/peft`` - an import-only stand-in for ``peft``, which the
  reference imports at module level (``wavelet/trainer/model.py:17``) but
  which is not installed.  The dense configuration sets ``lora: null``, so no
  ``peft`` function runs.
* a local Hugging Face model directory for the Qwen2.5-7B shape: a
  ``config.json`` for ``Qwen2ForCausalLM``, a word-level tokenizer with a
  ChatML template (the fake data source renders ``tok0 tok1 ...`` prompts
  through the tokenizer's chat template, ``wavelet/data/sft.py:195-212``) and a
  ``model.safetensors`` whose tensors are written as a sparse all-zero file.
  After ``setup()`` every parameter is re-initialised in place on the device
  (matrices N(0, 0.02), norm weights 1, biases 0), so the trainer starts from
  random-init weights as the benchmark configuration asks, without writing
  15 GB of random bytes to disk first.

Timing mirrors the native arm: W warm-up optimizer steps, then K steps
bracketed by a barrier and ``torch.cuda.synchronize()`` on both sides and
timed with CUDA events on the current stream, max over ranks.  The stock loop
is end to end by construction (host data loader -> pinned host batch -> device
copy in ``_prepare_batch`` -> step -> ``loss.item()``), so the e2e figure is
the host wall clock of the same K steps, and the bytes are counted from one
batch of the real data loader.
"""

from __future__ import annotations

import json
import os
import struct
import sys
import tempfile
import time
import zlib
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_ROOT = HERE / "_ref"
SHIMS = HERE / "shims"

# Qwen2.5-7B shape (the headline dense SFT configuration).
QWEN25_7B = {
    "architectures": ["Qwen2ForCausalLM"],
    "model_type": "qwen2",
    "vocab_size": 152064,
    "hidden_size": 3584,
    "intermediate_size": 18944,
    "num_hidden_layers": 28,
    "num_attention_heads": 28,
    "num_key_value_heads": 4,
    "max_position_embeddings": 32768,
    "rope_theta": 1000000.0,
    "rms_norm_eps": 1e-6,
    "hidden_act": "silu",
    "tie_word_embeddings": False,
    "use_sliding_window": False,
    "sliding_window": None,
    "max_window_layers": 28,
    "attention_dropout": 0.0,
    "initializer_range": 0.02,
    "use_cache": False,
    "bos_token_id": 0,
    "eos_token_id": 2,
    "pad_token_id": 0,
    "torch_dtype": "bfloat16",
}

CHATML = (
    "{% for message in messages %}"
    "{{ '<|im_start|>' + message['role'] + '\n' + message['content'] + '<|im_end|>' + '\n' }}"
    "{% endfor %}"
    "{% if add_generation_prompt %}{{ '<|im_start|>assistant\n' }}{% endif %}"
)


def unavailable_reason() -> str | None:
    if not (REF_ROOT / "wavelet" / "__init__.py").is_file():
        return (f"reference package missing: {REF_ROOT / 'wavelet'} does not exist "
                "(copy the reference's wavelet/ package there; pip install fails offline: no hatchling)")
    return None


def _write_tokenizer(model_dir: Path, n_words: int) -> None:
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace

    specials = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]
    words = ["system", "user", "assistant"] + [f"tok{i}" for i in range(n_words)]
    vocab = {t: i for i, t in enumerate(specials + words)}
    tok = Tokenizer(WordLevel(vocab=vocab, unk_token="<|endoftext|>"))
    tok.pre_tokenizer = Whitespace()
    tok.add_special_tokens(specials)
    tok.save(str(model_dir / "tokenizer.json"))
    (model_dir / "tokenizer_config.json").write_text(json.dumps({
        "tokenizer_class": "PreTrainedTokenizerFast",
        "model_max_length": 131072,
        "bos_token": None,
        "eos_token": "<|im_end|>",
        "pad_token": "<|endoftext|>",
        "unk_token": "<|endoftext|>",
        "chat_template": CHATML,
    }))
    (model_dir / "special_tokens_map.json").write_text(json.dumps({
        "eos_token": "<|im_end|>", "pad_token": "<|endoftext|>", "unk_token": "<|endoftext|>"}))


def _write_sparse_safetensors(model_dir: Path, arch: dict) -> None:
    """Writes ``model.safetensors`` with the model's tensor names and shapes and
    all-zero data, as a sparse file (the header is real; the data region is a
    hole, so the file costs no disk blocks and reads back as zeros)."""
    import torch
    from transformers import AutoConfig, AutoModelForCausalLM

    cfg = AutoConfig.from_pretrained(str(model_dir))
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16)
    header: dict = {"__metadata__": {"format": "pt"}}
    off = 0
    for name, t in model.state_dict().items():
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": "BF16", "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    path = model_dir / "model.safetensors"
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        f.truncate(8 + len(raw) + off)


def make_model_dir(root: Path, arch: dict, seq_len: int) -> Path:
    model_dir = root / "model"
    model_dir.mkdir(parents=True, exist_ok=True)
    done = model_dir / ".complete"
    if done.exists():
        return model_dir
    (model_dir / "config.json").write_text(json.dumps(arch))
    (model_dir / "generation_config.json").write_text(json.dumps({"bos_token_id": 0, "eos_token_id": 2}))
    _write_tokenizer(model_dir, seq_len + 16)
    _write_sparse_safetensors(model_dir, arch)
    done.write_text("ok")
    return model_dir


def _reinit_parameters(model, seed: int) -> None:
    """Random-init in place: N(0, 0.02) matrices, unit norm weights, zero biases.
    Each parameter draws from a generator seeded by its name, so replicas of a
    parameter on different ranks (tensor-parallel replication) agree."""
    import torch

    try:
        from torch.distributed.tensor import DTensor
    except Exception:  # pragma: no cover
        DTensor = ()
    with torch.no_grad():
        for name, p in model.named_parameters():
            local = p.to_local() if isinstance(p, DTensor) else p
            if local.numel() == 0:
                continue
            if name.endswith("norm.weight") or "layernorm" in name:
                local.fill_(1.0)
            elif name.endswith(".bias"):
                local.zero_()
            else:
                g = torch.Generator(device=local.device)
                g.manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
                tmp = torch.empty(local.shape, dtype=torch.float32, device=local.device)
                tmp.normal_(0.0, 0.02, generator=g)
                local.copy_(tmp)


def _batch_bytes(trainer) -> int:
    it = iter(trainer.dataloader)
    batch = next(it)
    n = 0
    for v in batch.values():
        if hasattr(v, "element_size"):
            n += v.numel() * v.element_size()
    return n


def run(args, clock_sampler_cls) -> int:
    reason = unavailable_reason()
    rank = int(os.environ.get("RANK", "0"))
    N = int(os.environ.get("WORLD_SIZE", "1"))
    if reason is not None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
        return 0
    sys.path.insert(0, str(REF_ROOT))
    sys.path.insert(1, str(SHIMS))

    import torch
    import torch.distributed as dist

    from wavelet.configs.config import SFTConfig
    from wavelet.monitor import setup_config_logger
    from wavelet.trainer.trainer import SFTTrainer
    from wavelet.utils.pathing import get_config_dir, validate_output_dir
    from wavelet.utils.serialization import dump_yaml

    arch = dict(QWEN25_7B)
    if getattr(args, "layers", None):
        arch["num_hidden_layers"] = arch["max_window_layers"] = args.layers
    if getattr(args, "ref_arch_overrides", None):
        arch.update(args.ref_arch_overrides)
    S = args.seq_len or 4096
    tp = args.tp
    dp = N // tp
    mb_per_dp_rank = args.micro_batches or 8 * tp
    global_batch = mb_per_dp_rank * dp
    total_steps = args.warmup + args.steps
    port = os.environ.get("MASTER_PORT", "x")
    work = Path(os.environ.get("WAVELET_REF_WORKDIR", tempfile.gettempdir())) / f"wb_ref_sft_{port}"
    # every rank writes its own copy of the (sparse) model directory: no cross-rank file race
    model_dir = make_model_dir(work / f"rank{rank}", arch, S)
    out_dir = work / "out"
    device_type = "cuda" if torch.cuda.is_available() else "cpu"

    cfg_dict = {
        "model": {
            "name": str(model_dir),
            "torch_dtype": "bfloat16",
            "attn_implementation": args.ref_attn,
            "activation_checkpointing": (None if args.activation_checkpointing == "none" else {"mode": "full"}),
        },
        "data": {
            "source": "fake",
            "batch_size": global_batch,
            "micro_batch_size": 1,
            "seq_len": S,
            "pack_function": "cat",
            "shuffle": False,
            "max_examples": global_batch * (total_steps + args.steps + 4),
            "num_workers": 0,
        },
        "optim": {"type": "adamw", "implementation": "fused", "lr": 1e-5, "weight_decay": 0.0,
                  "betas": [0.9, 0.999]},
        "lora": None,
        "ckpt": None,
        "max_grad_norm": 1.0,
        "max_steps": total_steps + args.steps + 2,
        "seed": 1234,
        "fsdp": {"enabled": True, "impl": "fsdp2", "tp": tp,
                 "backend": "auto" if device_type == "cuda" else "gloo"},
        "monitor": {"wandb": {"enabled": False}},
        "output_dir": str(out_dir),
        "clean_output_dir": True,
        "dist_timeout_seconds": 900,
    }
    config = SFTConfig.model_validate(cfg_dict)
    if rank == 0:
        validate_output_dir(config.output_dir, resuming=False, clean=True, protected_paths=())
        dump_yaml(get_config_dir(config.output_dir) / "sft.yaml", config.model_dump(mode="json", exclude_none=True))
    setup_config_logger("sft", config)
    trainer = SFTTrainer(config)
    try:
        trainer.setup()
    except Exception as exc:  # a blocker inside the stock path: report it, do not mask it
        import traceback

        tb = traceback.extract_tb(exc.__traceback__)
        where = f"{tb[-1].filename}:{tb[-1].lineno}" if tb else "?"
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                f"stock SFTTrainer.setup() failed at {where}: {type(exc).__name__}: {exc}")[:600],
                "config": {"parallelism": f"dp{dp}" + (f"xtp{tp}" if tp > 1 else "")}}), flush=True)
        if dist.is_initialized():
            dist.destroy_process_group()
        return 0
    _reinit_parameters(trainer.model, seed=1234)
    h2d = _batch_bytes(trainer) * trainer.accumulation_steps
    dev = trainer.world.device
    distributed = dist.is_initialized() and dist.get_world_size() > 1

    trainer.train_until(args.warmup)

    sampler = clock_sampler_cls(dev.index if dev.index is not None else 0) if (rank == 0 and device_type == "cuda") else None
    if sampler:
        sampler.start()
    if distributed:
        dist.barrier()
    if device_type == "cuda":
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
    t0 = time.perf_counter()
    trainer.train_until(total_steps)
    if device_type == "cuda":
        end.record()
        torch.cuda.synchronize()
    t1 = time.perf_counter()
    if distributed:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    dev_ms = (start.elapsed_time(end) if device_type == "cuda" else (t1 - t0) * 1000.0) / args.steps
    wall_ms = (t1 - t0) * 1000.0 / args.steps
    t = torch.tensor([dev_ms, wall_ms], dtype=torch.float64, device=dev)
    if distributed:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, wall_ms = float(t[0]), float(t[1])
    tokens_per_step = global_batch * S
    value = tokens_per_step / (dev_ms / 1000.0)
    loaded = sorted({m.__file__ for m in list(sys.modules.values())
                     if getattr(m, "__file__", None) and "wavelet_b200" in str(m.__file__)})
    if rank == 0:
        rec = {
            "impl": "reference",
            "metric": "SFT tok/s (Qwen2.5-7B-shape dense SFT, bf16)",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": N,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": dev_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (reference fake source: tok0..tokS prompt/completion rendered through a ChatML "
                    "word-level tokenizer, cat-packed to seq_len; random-init weights re-drawn on the device)",
            "config": {
                "model": "Qwen2.5-7B-shape" + (f" ({args.layers} layers: INVALID debug run)" if args.layers else ""),
                "global_batch": global_batch,
                "seq_len": S,
                "micro_batch": 1,
                "grad_accum": trainer.accumulation_steps,
                "parallelism": f"dp{dp}" + (f"xtp{tp}" if tp > 1 else ""),
                "optimizer": "torch fused AdamW on FSDP2-sharded bf16 parameters (reference default)",
                "attention": args.ref_attn,
                "activation_checkpointing": args.activation_checkpointing,
                "stack": "reference wavelet (baseline/_ref) SFTTrainer: FSDP2 + NCCL + cuBLAS via torch; "
                         "peft import shim (lora: null, never called)",
                "l2": "inputs larger than L2 (15 GB of weights per step)",
            },
            "gpu_launches": None,
            "clocks": clocks,
            "e2e": {
                "value": tokens_per_step / (wall_ms / 1000.0),
                "unit": "tokens/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4 * trainer.accumulation_steps,
                "ms_per_step": wall_ms,
                "note": "host wall clock of the same K stock-loop steps (host data loader, pinned batch, "
                        "device copy, step, loss.item())",
            },
            "native_modules_imported": loaded,
        }
        print(json.dumps(rec), flush=True)
    if dist.is_initialized():
        dist.destroy_process_group()
    return 0
