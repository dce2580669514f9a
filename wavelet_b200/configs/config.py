"""Pydantic configuration schema.

The YAML surface is the reference's (wavelet/configs/config.py): the same
section and key names, defaults and legacy spellings, so an existing
``sft.yaml`` / ``rl.yaml`` loads unchanged.  Unknown keys are rejected
(``extra="forbid"``).  Keys that configure vLLM in the reference
(``inference.vllm.*``) configure the native generator here: memory budget,
context limit, parallel sizes and logprob/sampling-mask behaviour keep their
meaning.
"""

from __future__ import annotations

from pathlib import Path
from typing import Annotated, Any, Literal

from pydantic import AliasChoices, BaseModel, ConfigDict, Field, SecretStr, model_validator

VERIFIER_ROLLOUT_FUNCTION = "wavelet.orchestrator.verifiers:generate_rollouts"
# every value of orchestrator.custom_rollout_function that selects verifiers-package rollouts
VERIFIER_ROLLOUT_FUNCTIONS = (VERIFIER_ROLLOUT_FUNCTION, "wavelet.orchestrator.verifiers:generate_and_score", "verifiers")


class ConfigModel(BaseModel):
    """Base of every config section: misspelled or unknown keys are errors."""

    model_config = ConfigDict(extra="forbid")


# ======================================================================= model
DEFAULT_LORA_TARGET_MODULES = [
    "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj",
    "experts", "fc1_latent_proj", "fc2_latent_proj",
]

LORA_RANK_CAPACITIES = (8, 16, 32, 64, 128, 256, 320, 512)


def resolve_lora_rank_capacity(rank: int) -> int:
    """Smallest served LoRA rank bucket that holds ``rank``."""
    for cap in LORA_RANK_CAPACITIES:
        if rank <= cap:
            return cap
    raise ValueError(f"LoRA rank {rank} exceeds the maximum served capacity {LORA_RANK_CAPACITIES[-1]}.")


class ActivationOffloadingConfig(ConfigModel):
    pin_memory: bool = True


class LoRAConfig(ConfigModel):
    rank: int = Field(default=16, ge=1)
    alpha: float = Field(default=32.0, ge=0.0)
    dropout: float = Field(default=0.0, ge=0.0, le=1.0)
    optimization_dtype: Literal["model", "float32"] = "model"
    target_modules: list[str] = Field(default_factory=lambda: list(DEFAULT_LORA_TARGET_MODULES))
    modules_to_save: list[str] = Field(default_factory=list)

    @model_validator(mode="after")
    def _no_modules_to_save(self):
        if self.modules_to_save:
            raise ValueError("lora.modules_to_save is not supported: the adapters train LoRA factors only "
                             "(train the full model for modules that must be updated)")
        return self


class ActivationCheckpointingConfig(ConfigModel):
    mode: Literal["full", "selective"] = "full"
    freq: int = Field(default=1, ge=1)
    targets: list[str] | None = None

    @model_validator(mode="after")
    def _targets(self):
        if self.mode == "full" and self.targets is not None:
            raise ValueError("activation_checkpointing.targets is only valid in selective mode.")
        if self.targets is not None and any(not t.strip() for t in self.targets):
            raise ValueError("activation_checkpointing.targets cannot contain blank names.")
        return self


class VLMConfig(ConfigModel):
    vision_encoder_attr: str = "model.visual"
    freeze_vision_encoder: bool = True


class ModelConfig(ConfigModel):
    name: str = "Qwen/Qwen3-0.6B"
    adapter_path: Path | None = None
    chat_template: str | None = None
    trust_remote_code: bool = False
    vlm: VLMConfig | None = None
    experts_implementation: Literal["eager", "grouped_mm"] | None = None
    torch_dtype: Literal["auto", "float32", "float16", "bfloat16"] = "bfloat16"
    attn_implementation: Literal["auto", "flash_attention_2", "flash_attention_3", "sdpa", "eager"] = "auto"
    load_in_4bit: bool = False
    kbit_cast_non_quantized_to_float32: bool = True
    activation_checkpointing: ActivationCheckpointingConfig | None = ActivationCheckpointingConfig()
    meta_device_init: bool = False
    matmul_precision: Literal["highest", "high", "medium"] = "high"
    fused_lora_mlp: bool = False
    fused_lora_qkv: bool = False
    fused_lora_o: bool = False
    fused_lm_head_token_chunk_size: int | Literal["auto", "disabled"] = "disabled"
    smart_gc: bool = False
    compile: bool = False
    compile_fullgraph: bool = False
    freeze_moe_router: bool = False
    moe_router_dtype: Literal["float32", "none"] = "none"
    # Native-only: random initialisation instead of loading weights (synthetic
    # benchmarks), and overrides of the architecture fields.
    random_init: bool = False
    arch_overrides: dict[str, Any] = Field(default_factory=dict)

    @model_validator(mode="after")
    def _checks(self):
        if self.load_in_4bit and self.experts_implementation == "grouped_mm":
            raise ValueError("model.experts_implementation='grouped_mm' requires unquantized expert weights")
        if self.compile_fullgraph and not self.compile:
            raise ValueError("model.compile_fullgraph requires model.compile=true.")
        if self.smart_gc and self.activation_checkpointing is None:
            raise ValueError("model.smart_gc requires model.activation_checkpointing.")
        if self.smart_gc and self.activation_checkpointing != ActivationCheckpointingConfig():
            raise ValueError("model.smart_gc owns checkpoint placement and only composes with the default full mode.")
        return self


# ======================================================================== data
class LossMaskConfig(ConfigModel):
    system: bool = False
    user: bool = False
    assistant: bool = True
    tool: bool = False


class TrainingDataConfig(ConfigModel):
    source: Literal["local", "hf", "fake"] = "local"
    path: Path | list[Path] = Path("outputs/data.jsonl")
    hf_name: str | None = None
    hf_subsets: list[str] | None = None
    hf_splits: list[str] | None = None
    probabilities: list[float] | None = None
    stopping_strategy: Literal["first_exhausted", "all_exhausted"] = "first_exhausted"
    batch_size: int = Field(default=4, ge=1)
    micro_batch_size: int = Field(default=1, ge=1)
    num_workers: int = Field(default=0, ge=0)
    pin_memory: bool = True
    seq_len: int = Field(default=128, ge=8)
    shuffle: bool = True
    seed: int = 0
    max_examples: int | None = Field(default=None, ge=1)
    fake_vocab_size: int = Field(default=32000, ge=8)
    fake_length: Literal["fixed", "variable"] = "fixed"
    fake_input_ids: Literal["random", "increasing"] = "random"
    prompt_column: str = "prompt"
    completion_column: str = "completion"
    messages_column: str = "messages"
    system_prompt: str | None = None
    merge_messages_thinking: bool = False
    tools_column: str = "tools"
    chat_template_kwargs_column: str = "chat_template_kwargs"
    loss_mask: LossMaskConfig = LossMaskConfig()

    @model_validator(mode="after")
    def _source(self):
        if self.batch_size % self.micro_batch_size != 0:
            raise ValueError("batch_size must be divisible by micro_batch_size")
        if self.hf_subsets is not None and self.hf_splits is not None and len(self.hf_subsets) != len(self.hf_splits):
            raise ValueError("hf_subsets and hf_splits must have the same length")
        if self.source == "hf" and self.hf_name is None:
            raise ValueError("hf_name is required when data.source='hf'")
        if self.source == "local" and self.hf_name is not None:
            raise ValueError("hf_name is only valid when data.source='hf'")
        return self


class DataConfig(TrainingDataConfig):
    path: Path | list[Path] = Path("outputs/unsloth_math_data/sft_train.jsonl")
    pack_function: Literal["pad", "cat"] = "pad"
    # Native-only: fraction range of each fake sequence treated as prompt
    # (loss-masked), e.g. [0.1, 0.4] for the 7B benchmark.
    fake_prompt_fraction: tuple[float, float] = (0.0, 0.0)


class SFTValConfig(ConfigModel):
    interval: int = Field(default=50, ge=1)
    eval_on_start: bool = False
    data: DataConfig


# =================================================================== optimizer
class OptimizerConfig(ConfigModel):
    type: Literal["adamw", "adamw_8bit", "paged_adamw_8bit", "adam", "adam_8bit", "sgd", "sign_sgd", "muon"] = "adamw"
    implementation: Literal["for-loop", "foreach", "fused"] = "fused"
    lr: float = Field(default=1e-3, gt=0.0)
    weight_decay: float = Field(default=0.0, ge=0.0)
    momentum: float = Field(default=0.9, ge=0.0)
    nesterov: bool = True
    betas1: float = Field(default=0.9, ge=0.0)
    betas2: float = Field(default=0.999, ge=0.0)
    cpu_offload: bool = False
    muon_momentum: float = Field(default=0.95, ge=0.0, lt=1.0)

    @model_validator(mode="before")
    @classmethod
    def _betas(cls, value):
        if not isinstance(value, dict) or "betas" not in value:
            return value
        v = dict(value)
        b = v.pop("betas")
        if not isinstance(b, (list, tuple)) or len(b) != 2:
            raise ValueError("optim.betas must be a 2-item list like [0.9, 0.999]")
        for name, beta in (("betas1", b[0]), ("betas2", b[1])):
            if name in v and v[name] != beta:
                raise ValueError(f"optim.betas and optim.{name} disagree; set only one of them.")
            v[name] = beta
        return v

    @model_validator(mode="after")
    def _offload(self):
        if self.cpu_offload and self.type == "sign_sgd":
            raise ValueError("optim.cpu_offload has no effect on stateless sign_sgd.")
        if self.cpu_offload and self.type in {"adamw_8bit", "paged_adamw_8bit", "adam_8bit"}:
            raise ValueError("optim.cpu_offload supports the native optimizers only.")
        return self


class SchedulerConfig(ConfigModel):
    type: Literal["constant", "linear", "cosine", "sqrt"] = "constant"
    warmup_ratio: float = Field(default=0.0, ge=0.0, le=1.0)
    warmup_steps: int | None = Field(default=None, ge=0)
    decay_steps: int | None = Field(default=None, ge=1)
    min_lr: float = Field(default=0.0, ge=0.0)
    min_lr_factor: float | None = Field(default=None, ge=0.0, le=1.0)
    decay_ratio: float = Field(default=1.0, ge=0.0, le=1.0)


class GCConfig(ConfigModel):
    interval: int = Field(default=50, ge=1)


class ProfilerConfig(ConfigModel):
    start_step: int = Field(default=1, ge=1)
    end_step: int = Field(default=1, ge=1)
    trace_path: Path | None = None
    record_shapes: bool = True
    profile_memory: bool = True

    @model_validator(mode="after")
    def _range(self):
        if self.end_step < self.start_step:
            raise ValueError("profiler.end_step must be >= profiler.start_step")
        return self


class MemoryProfilerConfig(ConfigModel):
    interval: int = Field(default=1, ge=1)
    max_entries: int = Field(default=100_000, ge=1)
    output_dir: Path | None = None


class CheckpointConfig(ConfigModel):
    interval: int | None = Field(default=None, ge=1)
    resume_step: int | None = None
    resume_dir: Path | None = None
    skip_optimizer: bool = False
    skip_scheduler: bool = False
    skip_dataloader: bool = False
    skip_progress: bool = False
    keep_last: int = Field(default=2, ge=1)
    keep_interval: int | None = Field(default=None, ge=1)
    mode: Literal["disabled", "async", "async_with_pinned_mem"] = "disabled"
    output_dir: Path | None = None

    @property
    def is_resuming(self) -> bool:
        return self.resume_step is not None or self.resume_dir is not None


class FSDPConfig(ConfigModel):
    enabled: bool = False
    impl: Literal["fsdp1", "fsdp2"] = "fsdp1"
    backend: Literal["auto", "gloo", "nccl", "hybrid"] = "auto"
    dp_replicate: int = Field(default=1, ge=1)
    dp_shard: int = -1
    cp: int = Field(default=1, ge=1)
    tp: int = Field(default=1, ge=1)
    ep: int = Field(default=1, ge=1)
    cpu_offload: bool = False
    reshard_after_forward: bool = True
    # ZeRO-3: the bf16 weights are sharded over the data-parallel (x context)
    # group too and gathered one decoder layer at a time, again in backward
    # (FSDP2 with reshard_after_forward); off: every rank keeps the full bf16
    # weights and only the fp32 optimizer state is sharded
    shard_params: bool = False
    # how expert-parallel token copies move on one CUDA node: fused row kernels
    # over peer memory ("fabric") or variable-split NCCL all-to-alls ("nccl")
    ep_dispatch: Literal["fabric", "nccl"] = "fabric"
    # expert-parallel row buffers (fabric dispatch): unset = room for the worst
    # routing; a number = that many times the average (token, expert) copies
    # per rank (less memory; a layer whose routing needs more is an error)
    ep_capacity_factor: float | None = Field(default=None, ge=1.0)
    # how tensor-parallel partial sums are reduced on one CUDA node: GEMMs whose
    # epilogue stores into the peers' buffers ("fabric") or NCCL all-reduce
    tp_reduce: Literal["fabric", "nccl"] = "fabric"

    @model_validator(mode="after")
    def _checks(self):
        if self.impl == "fsdp1" and not self.reshard_after_forward:
            raise ValueError("fsdp.reshard_after_forward=false requires fsdp.impl='fsdp2'.")
        if self.ep > 1 and self.tp > 1:
            raise ValueError("fsdp.tp>1 cannot be combined with fsdp.ep>1.")
        bad = []
        if self.ep > 1 and (not self.enabled or self.impl != "fsdp2"):
            bad.append(f"fsdp.ep={self.ep}")
        if self.cp > 1 and (not self.enabled or self.impl != "fsdp2"):
            bad.append(f"fsdp.cp={self.cp}")
        if bad:
            raise ValueError(f"{', '.join(bad)} requires enabled FSDP2 (context and expert parallelism).")
        return self


class LogConfig(ConfigModel):
    level: Literal["debug", "info", "warning", "error", "critical"] = "info"
    log_every: int = Field(default=1, ge=1)
    json_console: bool = False
    json_file: bool = True


class WandbConfig(ConfigModel):
    enabled: bool = False
    project: str | None = None
    entity: str | None = None
    name: str | None = None
    group: str | None = None
    tags: list[str] | None = None
    mode: Literal["online", "offline", "disabled"] = "offline"
    init_timeout_seconds: float = Field(default=30.0, gt=0.0)
    offline_fallback: bool = True
    create_overview: bool = True


class SampleLogConfig(ConfigModel):
    enabled: bool = False
    interval: int = Field(default=10, ge=1)
    sample_ratio: float | None = Field(default=None, ge=0.0, le=1.0)
    max_samples: int | None = Field(default=None, ge=1)
    keep_last: int = Field(default=256, ge=1)


class MonitorConfig(ConfigModel):
    enabled: bool = True
    write_events: bool = True
    write_metrics_jsonl: bool = True
    write_metrics_csv: bool = True
    write_run_metadata: bool = True
    write_heartbeat: bool = True
    log_cuda_memory: bool = True
    log_disk_usage: bool = True
    wandb: WandbConfig = WandbConfig()
    samples: SampleLogConfig = SampleLogConfig()


class DeploymentConfig(ConfigModel):
    type: Literal["single_node", "multi_node"] = "single_node"
    num_train_nodes: int = Field(default=1, ge=1)
    num_inference_nodes: int = Field(default=0, ge=0)
    inference_replicas_per_node: int = Field(default=1, ge=1)
    gpus_per_node: int = Field(default=1, ge=1)
    trainer_master_port: int = Field(default=29500, ge=1, le=65535)

    @model_validator(mode="after")
    def _nodes(self):
        total = self.num_train_nodes + self.num_inference_nodes
        if self.inference_replicas_per_node != 1 and self.num_inference_nodes == 0:
            raise ValueError("Inference replicas per node require inference nodes.")
        if self.type == "single_node" and total != 1:
            raise ValueError("deployment.type='single_node' requires exactly one train node and no inference nodes.")
        if self.type == "multi_node" and total < 2:
            raise ValueError("deployment.type='multi_node' requires at least two total nodes.")
        return self


_MANAGED_SLURM = {
    "--job-name", "--nodes", "--ntasks-per-node", "--gpus-per-node", "--output", "--error", "--partition",
    "--account", "--qos", "--time", "--constraint", "--reservation", "--nodelist", "--exclude",
    "--cpus-per-task", "--mem", "--exclusive",
}


class SlurmConfig(ConfigModel):
    job_name: str = Field(default="wavelet", min_length=1)
    project_dir: Path = Path(".")
    partition: str | None = None
    account: str | None = None
    qos: str | None = None
    time_limit: str | None = None
    constraint: str | None = None
    reservation: str | None = None
    nodelist: str | None = None
    exclude: str | None = None
    cpus_per_task: int | None = Field(default=None, ge=1)
    memory: str | None = None
    inference_cpus_per_replica: int = Field(default=1, ge=1)
    inference_memory_per_replica: str | None = Field(default=None, min_length=1)
    exclusive: bool = False
    shared_fs: bool = True
    setup_commands: list[str] = Field(default_factory=list)
    python_command: str = "python"
    extra_directives: list[str] = Field(default_factory=list)

    @model_validator(mode="after")
    def _shell(self):
        for name in ("job_name", "partition", "account", "qos", "time_limit", "constraint", "reservation",
                     "nodelist", "exclude", "memory", "inference_memory_per_replica", "python_command"):
            v = getattr(self, name)
            if v is not None and any(c in v for c in "\r\n\0"):
                raise ValueError(f"slurm.{name} cannot contain control characters.")
        if not self.python_command.strip():
            raise ValueError("slurm.python_command cannot be blank.")
        for d in self.extra_directives:
            if not d.startswith("--") or any(c in d for c in "\r\n\0"):
                raise ValueError("slurm.extra_directives entries must be single-line options beginning with '--'.")
            if d.split("=", 1)[0].split(maxsplit=1)[0] in _MANAGED_SLURM:
                raise ValueError(f"slurm.extra_directives cannot override managed option {d}.")
        return self


# ===================================================================== trainer
class TrainerConfig(ConfigModel):
    model: ModelConfig = ModelConfig()
    optim: OptimizerConfig = OptimizerConfig()
    scheduler: SchedulerConfig = SchedulerConfig()
    gc: GCConfig | None = GCConfig()
    profiler: ProfilerConfig | None = None
    memory_profiler: MemoryProfilerConfig | None = None
    max_grad_norm: float = Field(default=1.0, ge=0.0)
    loss_impl: Literal["liger", "torch", "liger_fused"] = "torch"
    ckpt: CheckpointConfig | None = None
    lora: LoRAConfig | None = LoRAConfig()
    log: LogConfig = LogConfig()
    monitor: MonitorConfig = MonitorConfig()
    fsdp: FSDPConfig = FSDPConfig()
    deployment: DeploymentConfig = DeploymentConfig()
    slurm: SlurmConfig | None = None
    output_dir: Path = Path("outputs/train")
    clean_output_dir: bool = False
    dry_run: bool = False
    epochs: int = Field(default=1, ge=1)
    max_steps: int | None = Field(default=None, ge=0)
    seed: int = 0
    dist_timeout_seconds: int = Field(default=1800, ge=1)
    activation_offloading: ActivationOffloadingConfig | None = None

    @model_validator(mode="after")
    def _deploy(self):
        if self.deployment.type == "multi_node" and self.slurm is None:
            raise ValueError("deployment.type='multi_node' requires a slurm configuration.")
        if self.slurm is not None and self.deployment.type != "multi_node":
            raise ValueError("slurm requires deployment.type='multi_node'; use the normal launcher for a single-node run.")
        if self.slurm is not None and not self.slurm.shared_fs:
            raise ValueError("SLURM deployment currently requires slurm.shared_fs=true.")
        return self

    @property
    def checkpoint_output_dir(self) -> Path:
        if self.ckpt is not None and self.ckpt.output_dir is not None:
            return self.ckpt.output_dir
        return self.output_dir

    @model_validator(mode="after")
    def _fused_lora(self):
        fused = [n for n in ("fused_lora_mlp", "fused_lora_qkv", "fused_lora_o") if getattr(self.model, n)]
        if fused and self.lora is not None:
            if self.lora.dropout > 0.0:
                raise ValueError(f"model.{fused[0]} does not apply lora.dropout; set lora.dropout=0.")
            if self.lora.optimization_dtype != "model":
                raise ValueError(f"model.{fused[0]} needs lora.optimization_dtype='model'.")
        return self

    @model_validator(mode="after")
    def _cp(self):
        if self.fsdp.cp <= 1:
            return self
        if self.model.vlm is not None:
            raise ValueError("Context parallelism is not supported for VLM models.")
        if self.model.attn_implementation != "sdpa":
            raise ValueError("Context parallelism requires model.attn_implementation='sdpa'.")
        loss = getattr(self, "loss", None)
        if loss is not None and loss.normalization != "token":
            raise ValueError("Context parallelism requires loss.normalization='token'.")
        data = getattr(self, "data", None)
        if data is not None and data.seq_len % (2 * self.fsdp.cp) != 0:
            raise ValueError("Sequence length must be divisible by 2 * CP degree when CP is enabled.")
        return self

    @model_validator(mode="after")
    def _ckpt(self):
        c = self.ckpt
        if c is None:
            return self
        if c.resume_step is not None and c.resume_step < -1:
            raise ValueError("ckpt.resume_step must be >= -1")
        if c.resume_step is not None and c.resume_dir is not None:
            raise ValueError("ckpt.resume_step and ckpt.resume_dir are mutually exclusive")
        if c.resume_dir is not None and not c.resume_dir.name.removeprefix("checkpoint-").removeprefix("step-").isdigit():
            raise ValueError("ckpt.resume_dir must point to a step directory")
        skips = [n for n in ("skip_optimizer", "skip_scheduler", "skip_dataloader", "skip_progress") if getattr(c, n)]
        if skips and not c.is_resuming:
            raise ValueError(f"{', '.join('ckpt.' + n for n in skips)} require checkpoint resume")
        if c.mode != "disabled" and c.interval is None:
            raise ValueError("ckpt.interval is required when checkpointing is enabled")
        if c.mode == "disabled":
            explicit = [f"ckpt.{n}" for n, v in (("interval", c.interval), ("keep_interval", c.keep_interval),
                                                 ("output_dir", c.output_dir)) if v is not None]
            if explicit:
                raise ValueError(f"{', '.join(explicit)} set while ckpt.mode='disabled' would never write checkpoints.")
        return self


class SFTConfig(TrainerConfig):
    data: DataConfig = DataConfig()
    val: SFTValConfig | None = None
    output_dir: Path = Path("outputs/unsloth_math_sft")
    max_steps: int | None = Field(default=None, ge=1)

    @model_validator(mode="after")
    def _sft_deploy(self):
        if self.deployment.num_inference_nodes != 0:
            raise ValueError("SFT deployment does not use inference nodes.")
        return self


# ========================================================================== RL
class _LegacySampling(ConfigModel):
    @model_validator(mode="before")
    @classmethod
    def _max_tokens(cls, value):
        if not isinstance(value, dict) or "max_tokens" not in value:
            return value
        v = dict(value)
        legacy = v.pop("max_tokens")
        if v.get("max_completion_tokens", legacy) != legacy:
            raise ValueError("sampling.max_tokens and sampling.max_completion_tokens disagree; set only max_completion_tokens.")
        v["max_completion_tokens"] = legacy
        return v


class RLDataConfig(TrainingDataConfig):
    path: Path | list[Path] = Path("outputs/unsloth_math_data/rl_train.jsonl")
    pack_sequences: bool = False
    pad_to_multiple_of: int = Field(default=1, ge=1)
    advantage_column: str = "advantage"
    reward_column: str = "reward"
    inference_logprobs_column: str = "inference_logprobs"
    teacher_logprobs_column: str = "teacher_logprobs"
    sampling_mask_column: str = "sampling_mask"
    temperature_column: str = "temperature"
    ce_weight_column: str = "ce_weight"
    ref_kl_weight_column: str = "ref_kl_weight"
    metadata_column: str = "metadata"
    # Native-only: prompt length of the synthetic reverse-text task (data.source: fake)
    fake_prompt_len: int = Field(default=256, ge=1)

    @model_validator(mode="before")
    @classmethod
    def _legacy_cols(cls, value):
        if not isinstance(value, dict) or "reference_logprobs_column" not in value:
            return value
        v = dict(value)
        legacy = v.pop("reference_logprobs_column")
        if v.get("inference_logprobs_column", legacy) != legacy:
            raise ValueError("data.reference_logprobs_column and data.inference_logprobs_column disagree.")
        v["inference_logprobs_column"] = legacy
        return v

    @model_validator(mode="after")
    def _rl_checks(self):
        if self.seq_len % self.pad_to_multiple_of != 0:
            raise ValueError("RL data.pad_to_multiple_of must divide data.seq_len.")
        if self.num_workers > 1:
            raise ValueError("RL data.num_workers must be 0 or 1 (rollout rows are pretokenized).")
        return self


class RLLossConfig(ConfigModel):
    type: Literal["dppo", "ipo", "icepop", "custom"] = "dppo"
    ratio_low: float = Field(default=0.2, gt=0.0, allow_inf_nan=False)
    ratio_high: float = Field(default=5.0, gt=0.0, allow_inf_nan=False)
    import_path: str | None = None
    kwargs: dict[str, Any] = Field(default_factory=dict)
    dppo_mask_high: float = Field(default=0.20, ge=0.0)
    dppo_mask_low: float = Field(default=0.20, ge=0.0)
    ipo_epsilon: float = Field(default=0.10, ge=0.0)
    kl_tau: float = Field(default=1e-3, ge=0.0)
    adv_tau: float = Field(default=1.0, ge=0.0)
    teacher_tau: float = Field(default=0.0, ge=0.0)
    normalization: Literal["token", "sequence"] = "token"

    @model_validator(mode="before")
    @classmethod
    def _legacy(cls, value):
        if not isinstance(value, dict):
            return value
        v = dict(value)
        if "advantage_scale" in v and "adv_tau" not in v:
            v["adv_tau"] = v.pop("advantage_scale")
        if v.get("type") == "custom":
            builtin = {"dppo_mask_high", "dppo_mask_low", "ipo_epsilon", "kl_tau", "adv_tau", "teacher_tau", "ratio_low", "ratio_high"}
            clash = sorted(builtin & v.keys())
            if clash:
                raise ValueError(f"Built-in loss fields cannot be set for a custom loss: {', '.join(clash)}.")
        return v

    @model_validator(mode="after")
    def _custom(self):
        if self.ratio_low > self.ratio_high:
            raise ValueError("loss.ratio_low must not exceed loss.ratio_high")
        if self.type == "custom":
            if not (self.import_path or "").strip():
                raise ValueError("Custom RL loss requires a non-empty import_path.")
        elif self.import_path is not None or self.kwargs:
            raise ValueError("loss.import_path and loss.kwargs are only valid when loss.type='custom'.")
        return self


class RLTransportConfig(ConfigModel):
    type: Literal["filesystem"] = "filesystem"
    rollout_filename: str = "rollouts.jsonl"
    queue_dir: Path | None = None
    poll_interval_seconds: float = Field(default=1.0, gt=0.0)
    idle_timeout_seconds: float | None = Field(default=None, gt=0.0)
    cleanup_consumed: bool = True
    keep_last_consumed: int = Field(default=2, ge=1)


class RLPolicyTransferConfig(ConfigModel):
    # "nccl" is the in-process device broadcast (fused reshard + cast kernels
    # over NVLink peer memory, NCCL as the fallback transport).
    type: Literal["filesystem", "nccl"] = "filesystem"
    policy_dir: Path | None = None
    adapter_name: str = "policy"
    adapter_id: int = Field(default=1, ge=1)
    poll_interval_seconds: float = Field(default=1.0, gt=0.0)
    idle_timeout_seconds: float | None = Field(default=None, gt=0.0)
    export_initial: bool = True
    export_every_steps: int = Field(default=1, ge=1)
    keep_last: int = Field(default=2, ge=2)
    lightweight_lora: bool = True
    nccl_host: str = "127.0.0.1"
    nccl_port: int = Field(default=29501, ge=1, le=65535)
    nccl_timeout_seconds: int = Field(default=600, ge=1)
    nccl_inference_world_size: int = Field(default=1, ge=1)
    nccl_rank_offset: int = Field(default=1, ge=1)
    nccl_dtype: Literal["model", "bfloat16", "float32"] = "bfloat16"
    # device transfer between processes of one node: push over peer memory
    # into `peer_slots` receive buffers per generator (2: the trainer never
    # waits; 1: half the generator memory, a load may copy twice); off or
    # across nodes: the NCCL broadcast
    peer: bool = True
    peer_slots: int = Field(default=2, ge=1, le=2)


class RLSamplingConfig(_LegacySampling):
    temperature: float = Field(default=1.0, ge=0.0)
    top_p: float = Field(default=1.0, gt=0.0, le=1.0)
    top_k: int = Field(default=-1, ge=-1)
    min_p: float = Field(default=0.0, ge=0.0, le=1.0)
    min_tokens: int = Field(default=0, ge=0)
    repetition_penalty: float = Field(default=1.0, gt=0.0)
    max_prompt_tokens: int | None = Field(default=None, ge=1)
    max_completion_tokens: int | None = Field(default=None, ge=1)
    do_sample: bool = True
    num_generations: int = Field(default=1, ge=1)
    seed: int | None = None
    extra_body: dict[str, Any] = Field(default_factory=dict)

    @model_validator(mode="after")
    def _native_sampler(self):
        if self.repetition_penalty != 1.0:
            raise ValueError("inference.sampling.repetition_penalty is not supported by the native sampler "
                             "(it would change the sampled distribution the RL losses correct for); use 1.0")
        return self


class RLEvalSamplingConfig(_LegacySampling):
    temperature: float | None = Field(default=None, ge=0.0)
    top_p: float | None = Field(default=None, gt=0.0, le=1.0)
    top_k: int | None = Field(default=None, ge=-1)
    min_p: float | None = Field(default=None, ge=0.0, le=1.0)
    min_tokens: int | None = Field(default=None, ge=0)
    repetition_penalty: float | None = Field(default=None, gt=0.0)
    max_completion_tokens: int | None = Field(default=None, ge=1)
    reasoning_effort: Literal["minimal", "low", "medium", "high"] | None = None
    seed: int | None = None
    extra_body: dict[str, Any] = Field(default_factory=dict)

    @model_validator(mode="after")
    def _native_sampler(self):
        if self.repetition_penalty not in (None, 1.0):
            raise ValueError("eval sampling repetition_penalty is not supported by the native sampler; use 1.0")
        return self

    def to_sampling_args(self) -> dict[str, Any]:
        args: dict[str, Any] = {"logprobs": True}
        extra = {**self.extra_body, "return_token_ids": True}
        for k in ("temperature", "top_p", "max_completion_tokens", "reasoning_effort", "seed"):
            if getattr(self, k) is not None:
                args[k] = getattr(self, k)
        for k in ("top_k", "min_p", "min_tokens", "repetition_penalty"):
            if getattr(self, k) is not None:
                extra[k] = getattr(self, k)
        args["extra_body"] = extra
        return args


class _NamedEnvConfig(ConfigModel):
    id: str
    name: str | None = None

    @property
    def resolved_name(self) -> str:
        return self.name or self.id.split("@", 1)[0]


class RLEvalEnvConfig(_NamedEnvConfig):
    args: dict[str, Any] = Field(default_factory=dict)
    sampling: RLEvalSamplingConfig = RLEvalSamplingConfig()
    num_examples: int = -1
    rollouts_per_example: int = Field(default=1, ge=1)
    interval: int = Field(default=100, ge=1)
    max_retries: int = Field(default=0, ge=0)


class RLEvalConfig(ConfigModel):
    resume: bool = False
    model_revision: str | None = None
    live_traces: bool = True
    env: list[RLEvalEnvConfig] = Field(default_factory=list)
    sampling: RLEvalSamplingConfig = RLEvalSamplingConfig()
    num_examples: int = -1
    rollouts_per_example: int = Field(default=1, ge=1)
    interval: int = Field(default=100, ge=1)
    max_retries: int = Field(default=0, ge=0)
    max_inflight_rollouts: int = Field(default=64, ge=1)
    background: bool = False
    cancel_on_new_policy: bool = True
    eval_base_model: bool = True
    final_eval: bool = True
    keep_last_rollout_sets: int = Field(default=2, ge=1)

    @model_validator(mode="after")
    def _env_defaults(self):
        group = self.sampling.model_dump()
        for env in self.env:
            if "sampling" not in env.model_fields_set:
                env.sampling = RLEvalSamplingConfig(**group)
            else:
                env.sampling = RLEvalSamplingConfig(**(group | env.sampling.model_dump(exclude_unset=True)))
            for n in ("num_examples", "rollouts_per_example", "interval", "max_retries"):
                if n not in env.model_fields_set:
                    setattr(env, n, getattr(self, n))
        names = [e.resolved_name for e in self.env]
        dup = {n for n in names if names.count(n) > 1}
        if dup:
            raise ValueError(f"Duplicate evaluation environment names: {dup}")
        return self


_MANAGED_ENGINE_ARGS = frozenset({
    "chat_template", "data_parallel_rpc_port", "data_parallel_size", "data_parallel_size_local", "dtype",
    "enable_auto_tool_choice", "enable_log_requests", "enable_lora", "enable_sleep_mode", "enforce_eager",
    "fully_sharded_loras", "generation_config", "gpu_memory_utilization", "hf_overrides", "host", "load_format",
    "logprobs_mode", "max_cpu_loras", "max_lora_rank", "max_loras", "max_model_len", "model", "additional_config",
    "port", "quantization", "reasoning_parser", "return_sampling_mask", "tensor_parallel_size", "tool_call_parser",
    "trust_remote_code", "worker_extension_cls",
})


class RLVLLMConfig(ConfigModel):
    """Generator settings (historically named after vLLM; served natively)."""

    server_backend: Literal["offline", "openai"] = "openai"
    gpu_memory_utilization: float = Field(default=0.35, gt=0.0, le=1.0)
    max_model_len: int | None = Field(default=None, ge=8)
    quantization: str | None = None
    load_format: str | None = None
    tensor_parallel_size: int = Field(default=1, ge=1)
    data_parallel_size: int = Field(default=1, ge=1)
    data_parallel_size_local: int | None = Field(default=None, ge=1)
    data_parallel_rpc_port: int | None = Field(default=None, ge=1, le=65535)
    enforce_eager: bool = False
    max_lora_rank: int | None = Field(default=None, ge=1)
    fully_sharded_loras: bool = False
    trust_remote_code: bool | None = None
    dtype: Literal["auto", "float32", "float16", "bfloat16"] | None = None
    tool_call_parser: str | None = "auto"
    reasoning_parser: str | None = "auto"
    enable_fp32_lm_head: bool = True
    enable_fp32_router_logits: bool = True
    use_generation_logprobs: bool = True
    return_sampling_mask: bool | None = None
    openai_batch_wait_seconds: float = Field(default=0.01, ge=0.0)
    openai_batch_min_size: int = Field(default=1, ge=1)
    openai_batch_max_wait_seconds: float = Field(default=0.01, ge=0.0)
    openai_batch_max_size: int | None = Field(default=None, ge=1)
    extra_args: dict[str, Any] = Field(default_factory=dict)
    # Native generator knobs
    max_num_seqs: int = Field(default=512, ge=1)
    kv_block_size: int = Field(default=64, ge=16)
    cuda_graphs: bool = True

    @model_validator(mode="after")
    def _extra(self):
        seen: set[str] = set()
        for k in self.extra_args:
            n = k.replace("-", "_")
            if not n.isidentifier():
                raise ValueError(f"inference.vllm.extra_args keys must be argument names; got {k!r}.")
            if n in _MANAGED_ENGINE_ARGS:
                raise ValueError(f"inference.vllm.extra_args cannot override managed argument {k!r}.")
            if n in seen:
                raise ValueError(f"inference.vllm.extra_args contains duplicate normalized key {n!r}.")
            seen.add(n)
        return self


class RLVLLMHTTPConfig(ConfigModel):
    host: str = "127.0.0.1"
    hosts: list[str] | None = None
    port: int = Field(default=8000, ge=1, le=65535)
    ports: list[int] | None = None
    request_timeout_seconds: float = Field(default=300.0, gt=0.0)
    startup_timeout_seconds: float = Field(default=300.0, gt=0.0)
    liveness_timeout_seconds: float = Field(default=10.0, gt=0.0)

    @model_validator(mode="after")
    def _endpoints(self):
        if self.hosts is not None and (not self.hosts or any(not h.strip() for h in self.hosts)):
            raise ValueError("inference.http.hosts must list at least one non-blank host.")
        if self.ports is None:
            return self
        if not self.ports:
            raise ValueError("inference.http.ports must list at least one port.")
        if any(not 1 <= p <= 65535 for p in self.ports):
            raise ValueError("inference.http.ports entry out of range.")
        if self.hosts is None and len(set(self.ports)) != len(self.ports):
            raise ValueError("inference.http.ports must be unique; replicas cannot share a port.")
        if self.hosts is not None and len(self.hosts) != len(self.ports):
            raise ValueError("inference.http.hosts and inference.http.ports must have the same number of entries.")
        return self


class RLInferenceConfig(ConfigModel):
    enabled: bool = True
    mode: Literal["passthrough", "vllm_http"] = "vllm_http"
    default_temperature: float = Field(default=1.0, gt=0.0)
    sampling: RLSamplingConfig = RLSamplingConfig()
    vllm: RLVLLMConfig = RLVLLMConfig()
    http: RLVLLMHTTPConfig = RLVLLMHTTPConfig()


class RLRewardConfig(ConfigModel):
    mode: Literal["passthrough", "reference_match", "math_format", "reverse_match", "environment"] = "passthrough"
    normalize_whitespace: bool = True
    case_sensitive: bool = True
    reasoning_end: str = "<end_working_out>"
    solution_start: str = "<SOLUTION>"
    solution_end: str = "</SOLUTION>"
    rescale_min: float | None = None
    rescale_max: float | None = None
    clamp_min: float | None = None
    clamp_max: float | None = None

    @model_validator(mode="after")
    def _post(self):
        if (self.rescale_min is None) != (self.rescale_max is None):
            raise ValueError("reward.rescale_min and reward.rescale_max must be set together")
        if self.rescale_min is not None and self.rescale_max <= self.rescale_min:
            raise ValueError("reward.rescale_max must be greater than reward.rescale_min")
        if self.clamp_min is not None and self.clamp_max is not None and self.clamp_max < self.clamp_min:
            raise ValueError("reward.clamp_max must be greater than or equal to reward.clamp_min")
        return self


class RLStateServerConfig(ConfigModel):
    enabled: bool = False
    host: str = "127.0.0.1"
    port: int = Field(default=8765, ge=1, le=65535)
    log_level: Literal["critical", "error", "warning", "info", "debug", "trace"] = "warning"
    cors_allow_origins: list[str] = Field(default_factory=lambda: ["*"])
    max_events: int = Field(default=2000, ge=100)


class TokensLengthPenaltyConfig(ConfigModel):
    type: Literal["tokens"] = "tokens"
    completion_weight: float = Field(default=1.0, ge=0.0)
    tool_response_weight: float = Field(default=1.0, ge=0.0)


class TurnsLengthPenaltyConfig(ConfigModel):
    type: Literal["turns"] = "turns"


class LinearLengthPenaltyConfig(ConfigModel):
    type: Literal["linear"] = "linear"
    num_output_tokens_weight: float = Field(default=0.25, ge=0.0, allow_inf_nan=False)
    num_input_tokens_weight: float = Field(default=0.1, ge=0.0, allow_inf_nan=False)
    num_turns_weight: float = Field(default=0.1, ge=0.0, allow_inf_nan=False)


class TruncationLengthPenaltyConfig(ConfigModel):
    type: Literal["truncation"] = "truncation"
    penalty: float = Field(default=1.0, ge=0.0, allow_inf_nan=False)


LengthPenaltyConfig = Annotated[
    TokensLengthPenaltyConfig | TurnsLengthPenaltyConfig | LinearLengthPenaltyConfig | TruncationLengthPenaltyConfig,
    Field(discriminator="type"),
]


class PassthroughAlgorithmConfig(ConfigModel):
    type: Literal["passthrough"] = "passthrough"


class RewardAlgorithmConfig(ConfigModel):
    type: Literal["reward"] = "reward"


class GRPOAlgorithmConfig(ConfigModel):
    type: Literal["grpo"] = "grpo"
    normalize_advantages: bool = False
    epsilon: float = Field(default=1e-6, gt=0.0)
    length_penalty: LengthPenaltyConfig | None = None

    @model_validator(mode="before")
    @classmethod
    def _lp(cls, v):
        if isinstance(v, dict) and isinstance(v.get("length_penalty"), str):
            v = dict(v)
            v["length_penalty"] = {"type": v["length_penalty"]}
        return v


class MaxRLAlgorithmConfig(ConfigModel):
    type: Literal["max_rl"] = "max_rl"


class RLTeacherConfig(ConfigModel):
    name: str = Field(min_length=1, validation_alias=AliasChoices("name", "model"))
    base_url: str = Field(min_length=1)
    api_key_var: str = Field(default="OPENAI_API_KEY", min_length=1)
    timeout_seconds: float = Field(default=120.0, gt=0.0)

    @property
    def model(self) -> str:
        return self.name


class OPDAlgorithmConfig(ConfigModel):
    type: Literal["opd"] = "opd"
    teacher: RLTeacherConfig


class OPSDAlgorithmConfig(ConfigModel):
    type: Literal["opsd"] = "opsd"
    demo_key: str = Field(default="demonstration", min_length=1)
    template: str = "Here is an example of an expert response:\n<demonstration>\n{demonstration}\n</demonstration>"

    @model_validator(mode="after")
    def _tpl(self):
        if "{demonstration}" not in self.template:
            raise ValueError("OPSD template must contain '{demonstration}'.")
        return self


class SFTDistillAlgorithmConfig(ConfigModel):
    type: Literal["sft"] = "sft"


AlgorithmScope = Literal["rollout", "group", "both"]


class CustomAlgorithmConfig(ConfigModel):
    type: Literal["custom"] = "custom"
    file: Path
    algorithm: str = Field(min_length=1)
    scope: AlgorithmScope
    kwargs: dict[str, Any] = Field(default_factory=dict)
    epsilon: float = Field(default=1e-6, gt=0.0)


RLAlgorithmConfig = Annotated[
    PassthroughAlgorithmConfig | RewardAlgorithmConfig | GRPOAlgorithmConfig | MaxRLAlgorithmConfig
    | OPDAlgorithmConfig | OPSDAlgorithmConfig | SFTDistillAlgorithmConfig | CustomAlgorithmConfig,
    Field(discriminator="type"),
]


class RLAdaptiveConcurrencyConfig(ConfigModel):
    min_inflight: int = Field(default=1, ge=1)
    max_inflight: int | None = Field(default=None, ge=1)
    initial_inflight: int | None = Field(default=None, ge=1)
    growth_factor_per_turnover: float = Field(default=1.2, gt=1.0)
    binding_fraction: float = Field(default=0.9, gt=0.0, le=1.0)
    growth_gate_polls: int = Field(default=3, ge=1)
    growth_kv_cache_usage: float = Field(default=0.6, ge=0.0, lt=1.0)
    soft_kv_cache_usage: float = Field(default=0.8, gt=0.0, lt=1.0)
    target_kv_cache_usage: float = Field(default=0.7, gt=0.0, lt=1.0)
    hard_kv_cache_usage: float = Field(default=0.9, gt=0.0, le=1.0)
    queue_ratio: float = Field(default=0.5, ge=0.0)
    queue_persistence_polls: int = Field(default=6, ge=1)
    queue_decrease_factor: float = Field(default=0.9, gt=0.0, lt=1.0)
    preemption_decrease_factor: float = Field(default=0.8, gt=0.0, lt=1.0)
    kv_trim_cooldown_polls: int = Field(default=6, ge=0)
    poll_interval_seconds: float = Field(default=5.0, gt=0.0)
    request_timeout_seconds: float = Field(default=5.0, gt=0.0)

    @model_validator(mode="after")
    def _bounds(self):
        if self.max_inflight is not None:
            if self.min_inflight > self.max_inflight:
                raise ValueError("concurrency.min_inflight must not exceed concurrency.max_inflight.")
            if self.initial_inflight is not None and self.initial_inflight > self.max_inflight:
                raise ValueError("concurrency.initial_inflight must not exceed concurrency.max_inflight.")
        if self.initial_inflight is not None and self.initial_inflight < self.min_inflight:
            raise ValueError("concurrency.initial_inflight must be at least concurrency.min_inflight.")
        if not (self.growth_kv_cache_usage < self.target_kv_cache_usage < self.soft_kv_cache_usage < self.hard_kv_cache_usage):
            raise ValueError("concurrency KV thresholds must satisfy growth < target < soft < hard.")
        return self


class RLStandardCurriculumSamplerConfig(ConfigModel):
    type: Literal["standard"] = "standard"


class RLDifficultyPoolConfig(ConfigModel):
    threshold: float = Field(allow_inf_nan=False)
    weight: float = Field(ge=0.0, allow_inf_nan=False)


def _default_pools() -> dict[str, RLDifficultyPoolConfig]:
    return {
        "hard": RLDifficultyPoolConfig(threshold=0.25, weight=0.2),
        "normal": RLDifficultyPoolConfig(threshold=0.75, weight=1.0),
        "easy": RLDifficultyPoolConfig(threshold=1.0, weight=0.2),
    }


class RLDifficultyPoolSamplerConfig(ConfigModel):
    type: Literal["difficulty_pool"] = "difficulty_pool"
    pools: dict[str, RLDifficultyPoolConfig] = Field(default_factory=_default_pools)
    seed: int = 42
    ema_alpha: float = Field(default=0.2, gt=0.0, le=1.0, allow_inf_nan=False)

    @model_validator(mode="after")
    def _pools(self):
        if not self.pools:
            raise ValueError("curriculum difficulty pools cannot be empty.")
        if not any(p.weight > 0 for p in self.pools.values()):
            raise ValueError("At least one curriculum difficulty pool must have positive weight.")
        th = [p.threshold for p in self.pools.values()]
        if len(th) != len(set(th)):
            raise ValueError("Curriculum difficulty pool thresholds must be unique.")
        return self


RLCurriculumSamplerConfig = Annotated[
    RLStandardCurriculumSamplerConfig | RLDifficultyPoolSamplerConfig, Field(discriminator="type")
]


class RLAdvRangeGateConfig(ConfigModel):
    type: Literal["advantage_range"] = "advantage_range"
    reject_min: float = Field(default=0.0, allow_inf_nan=False)
    reject_max: float = Field(default=0.0, allow_inf_nan=False)

    @model_validator(mode="after")
    def _rng(self):
        if self.reject_min > self.reject_max:
            raise ValueError("reject_min must be less than or equal to reject_max.")
        return self


RLCurriculumGateConfig = Annotated[RLAdvRangeGateConfig, Field(discriminator="type")]


class RLCurriculumConfig(ConfigModel):
    sampler: RLCurriculumSamplerConfig = Field(default_factory=RLStandardCurriculumSamplerConfig)
    gates: dict[str, RLCurriculumGateConfig] = Field(default_factory=dict)


class RLTrainEnvConfig(_NamedEnvConfig):
    id: str = Field(min_length=1)
    args: dict[str, Any] = Field(default_factory=dict)
    ratio: float = Field(default=1.0, gt=0.0, allow_inf_nan=False)
    data_path: Path | None = None
    sampling: RLSamplingConfig | None = None
    group_size: int | None = Field(default=None, ge=1)
    algo: RLAlgorithmConfig | None = None
    curriculum: RLCurriculumConfig | None = None


class RLOrchestratorConfig(ConfigModel):
    live_traces: bool = True
    enabled: bool = True
    custom_rollout_function: str | None = None
    verifier_env_id: str | None = None
    verifier_env_args: dict[str, Any] = Field(default_factory=dict)
    envs: list[RLTrainEnvConfig] = Field(default_factory=list)
    verifier_model: str | None = None
    verifier_base_url: str | list[str] | None = None
    verifier_api_key_var: str = "PRIME_API_KEY"
    verifier_client_type: Literal["openai_chat_completions", "openai_chat_completions_token"] = "openai_chat_completions"
    verifier_max_retries: int = Field(default=0, ge=0)
    verifier_timeout_seconds: float | None = Field(default=None, gt=0.0)
    verifier_max_total_completion_tokens: int = -1
    materialize_path: Path | None = None
    overwrite: bool = True
    examples_per_step: int | None = Field(default=None, ge=1)
    token_batch_size: int | None = Field(default=None, ge=1)
    rollouts_per_example: int | None = Field(default=None, ge=1)
    oversampling_factor: float = Field(default=1.0, ge=1.0)
    max_inflight_rollouts: int | None = Field(default=None, ge=1)
    concurrency: RLAdaptiveConcurrencyConfig | None = None
    curriculum: RLCurriculumConfig | None = None
    rollout_chunk_examples: int | None = Field(default=None, ge=1)
    batch_selection: Literal["groups", "rollouts"] = "groups"
    filter_zero_advantage: bool = True
    refill_zero_advantage: bool = True
    zero_advantage_max_retries: int = Field(default=8, ge=0)
    max_async_level: int = Field(default=0, ge=0)
    max_off_policy_steps: int = Field(default=0, ge=0)
    max_pending_rollout_chunks: int | None = Field(default=None, ge=1)
    tasks_per_minute: int | None = Field(default=None, ge=1)
    pipeline_status_interval_seconds: float = Field(default=30.0, gt=0.0)
    state_server: RLStateServerConfig = RLStateServerConfig()

    @property
    def uses_verifiers(self) -> bool:
        return self.custom_rollout_function in VERIFIER_ROLLOUT_FUNCTIONS

    @model_validator(mode="after")
    def _checks(self):
        if self.batch_selection == "rollouts" and self.examples_per_step is None:
            raise ValueError("batch_selection='rollouts' requires examples_per_step.")
        if self.batch_selection == "rollouts" and self.refill_zero_advantage:
            raise ValueError("batch_selection='rollouts' requires refill_zero_advantage=false.")
        if self.examples_per_step is not None and self.token_batch_size is not None:
            raise ValueError("Set only one of orchestrator.examples_per_step and orchestrator.token_batch_size.")
        if self.token_batch_size is not None and self.rollout_chunk_examples is not None:
            raise ValueError("orchestrator.rollout_chunk_examples cannot be combined with orchestrator.token_batch_size; "
                             "token batches are one dynamic chunk per optimizer step.")
        if self.token_batch_size is not None and self.batch_selection == "rollouts":
            raise ValueError("orchestrator.token_batch_size counts the tokens of whole groups; "
                             "use batch_selection='groups'.")
        if self.envs and self.verifier_env_id is not None:
            raise ValueError("Set orchestrator.envs or legacy orchestrator.verifier_env_id, not both.")
        if self.envs and self.verifier_env_args:
            raise ValueError("orchestrator.verifier_env_args cannot be combined with orchestrator.envs.")
        if self.envs and self.curriculum is not None:
            raise ValueError("orchestrator.curriculum cannot be combined with orchestrator.envs.")
        if any(e.curriculum is not None for e in self.envs):
            raise ValueError("per-environment curriculum (orchestrator.envs[].curriculum) is not supported; "
                             "environments mix by their ratio")
        names = [e.resolved_name for e in self.envs]
        dup = sorted({n for n in names if names.count(n) > 1})
        if dup:
            raise ValueError(f"Duplicate training environment names: {', '.join(dup)}.")
        if self.max_inflight_rollouts is not None and self.rollouts_per_example is not None:
            if self.max_inflight_rollouts < self.rollouts_per_example:
                raise ValueError("orchestrator.max_inflight_rollouts must be at least orchestrator.rollouts_per_example")
        if self.tasks_per_minute is not None and not self.uses_verifiers:
            raise ValueError("orchestrator.tasks_per_minute currently requires the Verifiers rollout source.")
        return self


PROTECTED_ROLE_ENV_VARS = frozenset({
    "CUDA_VISIBLE_DEVICES", "GROUP_RANK", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
    "RANK", "ROLE_NAME", "ROLE_RANK", "WORLD_SIZE",
})


class RLRoleEnvConfig(ConfigModel):
    common: dict[str, SecretStr] = Field(default_factory=dict)
    inference: dict[str, SecretStr] = Field(default_factory=dict)
    trainer: dict[str, SecretStr] = Field(default_factory=dict)
    orchestrator: dict[str, SecretStr] = Field(default_factory=dict)

    @model_validator(mode="after")
    def _vars(self):
        for role in ("common", "inference", "trainer", "orchestrator"):
            env = getattr(self, role)
            bad = sorted(PROTECTED_ROLE_ENV_VARS.intersection(env))
            if bad:
                raise ValueError(f"launcher.env_vars.{role} cannot set launcher-managed variables {bad}.")
            inv = sorted(n for n in env if not n or "=" in n or "\x00" in n)
            if inv:
                raise ValueError(f"launcher.env_vars.{role} contains invalid variable names: {inv}.")
            if any("\x00" in v.get_secret_value() for v in env.values()):
                raise ValueError(f"launcher.env_vars.{role} values cannot contain NUL bytes.")
        return self

    def for_role(self, role: str) -> dict[str, str]:
        merged = {**self.common, **getattr(self, role)}
        return {k: v.get_secret_value() for k, v in merged.items()}


class RLLauncherConfig(ConfigModel):
    mode: Literal["integrated", "process", "colocate", "colocate_sleep"] = "integrated"
    backend: Literal["local", "ray"] = "local"
    trainer_cuda_visible_devices: str | list[str] | None = None
    inference_cuda_visible_devices: str | list[str] | None = None
    trainer_num_processes: int = Field(default=1, ge=1)
    inference_num_replicas: int = Field(default=1, ge=1)
    ray_address: str | None = None
    ray_runtime_env: dict[str, Any] | None = None
    env_vars: RLRoleEnvConfig = RLRoleEnvConfig()
    poll_interval_seconds: float = Field(default=1.0, gt=0.0)
    colocate_memory_wait_timeout_seconds: float = Field(default=120.0, ge=0.0)
    colocate_memory_wait_poll_seconds: float = Field(default=0.5, gt=0.0)
    colocate_memory_wait_margin: float = Field(default=0.05, ge=0.0, le=0.5)


_LEGACY_ADVANTAGE_KEYS = ("advantage_mode", "normalize_group_advantages", "advantage_epsilon", "length_penalty")


def _normalize_algorithm(value: dict[str, Any]) -> dict[str, Any]:
    """Move legacy ``orchestrator.advantage_mode`` settings into ``algo``."""
    v = dict(value)
    orch = v.get("orchestrator")
    legacy: dict[str, Any] = {}
    if isinstance(orch, dict):
        orch = dict(orch)
        legacy = {k: orch.pop(k) for k in _LEGACY_ADVANTAGE_KEYS if k in orch}
        v["orchestrator"] = orch
    if "algo" in v:
        if legacy:
            raise ValueError(f"{', '.join('orchestrator.' + k for k in legacy)} cannot be combined with an explicit algo block.")
        algo = v["algo"]
        if isinstance(algo, dict) and "type" not in algo and ("file" in algo or "algorithm" in algo):
            v["algo"] = {"type": "custom", **algo}
        return v
    if not legacy:
        return v
    mode = legacy.get("advantage_mode")
    grpo_only = [k for k in legacy if k != "advantage_mode"]
    if mode != "group_reward" and grpo_only:
        raise ValueError("GRPO advantage settings only apply with orchestrator.advantage_mode='group_reward'.")
    if mode != "group_reward":
        v["algo"] = {"type": mode}
        return v
    lp = legacy.get("length_penalty")
    v["algo"] = {
        "type": "grpo",
        "normalize_advantages": legacy.get("normalize_group_advantages", False),
        "epsilon": legacy.get("advantage_epsilon", 1e-6),
        "length_penalty": {"type": lp} if isinstance(lp, str) else lp,
    }
    return v


def _normalize_opd_teacher(value: dict[str, Any]) -> dict[str, Any]:
    v = dict(value)
    algo = v.get("algo")
    teacher = v.get("teacher")
    if not isinstance(algo, dict) or algo.get("type") != "opd" or teacher is None:
        return v
    if algo.get("teacher") is not None:
        raise ValueError("Configure the OPD teacher only under algo.teacher.")
    v["algo"] = {**algo, "teacher": teacher}
    v.pop("teacher", None)
    return v


class RLConfig(TrainerConfig):
    data: RLDataConfig = RLDataConfig()
    loss: RLLossConfig = RLLossConfig()
    algo: RLAlgorithmConfig = PassthroughAlgorithmConfig()
    teacher: RLTeacherConfig | None = None
    orchestrator: RLOrchestratorConfig = RLOrchestratorConfig()
    eval: RLEvalConfig | None = None
    inference: RLInferenceConfig = RLInferenceConfig()
    reward: RLRewardConfig = RLRewardConfig()
    transport: RLTransportConfig = RLTransportConfig()
    policy_transfer: RLPolicyTransferConfig = RLPolicyTransferConfig()
    launcher: RLLauncherConfig = RLLauncherConfig()
    output_dir: Path = Path("outputs/unsloth_math_rl")
    max_steps: int | None = Field(default=None, ge=0)

    @model_validator(mode="before")
    @classmethod
    def _legacy_algo(cls, value):
        if not isinstance(value, dict):
            return value
        return _normalize_opd_teacher(_normalize_algorithm(value))

    @model_validator(mode="after")
    def _lora_capacity(self):
        req = self.inference.vllm.max_lora_rank
        if self.lora is not None:
            req = max(req or 0, self.lora.rank)
        if req is not None:
            self.inference.vllm.max_lora_rank = resolve_lora_rank_capacity(req)
        return self

    @model_validator(mode="after")
    def _rl_deploy(self):
        if self.deployment.type != "multi_node":
            return self
        if self.launcher.mode != "process" or self.launcher.backend != "local":
            raise ValueError("Multi-node RL requires launcher.mode='process' and launcher.backend='local'.")
        return self

    @model_validator(mode="after")
    def _algos(self):
        algos = [c for _, c in self.train_algorithm_configs()]
        has_sft = any(isinstance(c, SFTDistillAlgorithmConfig) for c in algos)
        if has_sft and not all(isinstance(c, SFTDistillAlgorithmConfig) for c in algos):
            raise ValueError("SFT distillation cannot be mixed with policy-sampled algorithms.")
        if has_sft and self.teacher is None:
            raise ValueError("algo.type='sft' requires a top-level teacher block.")
        if self.teacher is not None and not has_sft:
            raise ValueError("The top-level teacher block is only used by algo.type='sft'.")
        if self.orchestrator.concurrency is not None:
            self._check_concurrency()
        if self.orchestrator.envs:
            if not self.orchestrator.uses_verifiers:
                raise ValueError("orchestrator.envs requires the Verifiers rollout source.")
            if not self._async_process():
                raise ValueError("orchestrator.envs requires launcher.mode='process' and orchestrator.max_async_level>=1.")
        return self

    def _check_concurrency(self) -> None:
        o = self.orchestrator
        if not o.uses_verifiers:
            raise ValueError("orchestrator.concurrency currently requires the Verifiers rollout source.")
        if not self._async_process():
            raise ValueError("orchestrator.concurrency requires launcher.mode='process' and "
                             "orchestrator.max_async_level>=1.")
        group = max([o.rollouts_per_example or 1] + [e.group_size or o.rollouts_per_example or 1 for e in o.envs])
        limits = {"initial_inflight": o.concurrency.initial_inflight, "max_inflight": o.concurrency.max_inflight}
        small = [k for k, v in limits.items() if v is not None and v < group]
        if small:
            raise ValueError(f"orchestrator.concurrency limits must be at least rollouts_per_example={group}: "
                             f"{', '.join(small)}.")
        ceiling = o.max_inflight_rollouts
        big = [k for k, v in limits.items() if ceiling is not None and v is not None and v > ceiling]
        if big:
            raise ValueError(f"orchestrator.concurrency limits cannot exceed the explicit "
                             f"orchestrator.max_inflight_rollouts={ceiling}: {', '.join(big)}.")

    def _async_process(self) -> bool:
        return self.launcher.mode == "process" and self.orchestrator.max_async_level >= 1

    def resolved_train_sampling(self, env: RLTrainEnvConfig | None = None) -> RLSamplingConfig:
        if env is None or env.sampling is None:
            return self.inference.sampling
        vals = self.inference.sampling.model_dump()
        vals.update(env.sampling.model_dump(exclude_unset=True))
        return RLSamplingConfig.model_validate(vals)

    def train_sampling_configs(self) -> list[tuple[str, RLSamplingConfig]]:
        if not self.orchestrator.envs:
            return [("train", self.inference.sampling)]
        return [(e.resolved_name, self.resolved_train_sampling(e)) for e in self.orchestrator.envs]

    def sampling_mask_required(self) -> bool:
        """Whether truncated sampling needs its support set recorded."""
        cfg = self.inference.vllm.return_sampling_mask
        if cfg is not None:
            return cfg
        return any(s.top_p < 1.0 or s.top_k > 0 or s.min_p > 0.0 for _, s in self.train_sampling_configs())

    def train_algorithm_configs(self) -> list[tuple[str, Any]]:
        if not self.orchestrator.envs:
            return [("train", self.algo)]
        return [(e.resolved_name, e.algo or self.algo) for e in self.orchestrator.envs]
