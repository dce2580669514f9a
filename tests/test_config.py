"""Config schema and CLI loader behaviour (CPU)."""

import json
from pathlib import Path

import pytest
import yaml
from pydantic import ValidationError

from wavelet_b200.configs.config import RLConfig, SFTConfig
from wavelet_b200.utils.config import help_text, load_config, load_yaml, parse_argv

ROOT = Path(__file__).resolve().parents[1]


def test_examples_load():
    for p in sorted((ROOT / "examples").rglob("*.yaml")):
        data = load_yaml(p)
        schema = RLConfig if p.name.startswith("rl") else SFTConfig
        schema.model_validate(data)


def test_unknown_key_rejected():
    with pytest.raises(ValidationError):
        SFTConfig.model_validate({"optim": {"lrr": 1.0}})


def test_overrides_and_bools(tmp_path):
    f = tmp_path / "a.yaml"
    f.write_text("optim:\n  lr: 0.5\nmodel:\n  compile: false\n")
    cfg = load_config(SFTConfig, ["@", str(f), "--optim.lr", "0.25", "--model.compile", "--no-monitor.enabled",
                                  "--data.seq-len", "256", "--optim.betas", "[0.8, 0.9]"])
    assert cfg.optim.lr == 0.25
    assert cfg.model.compile is True
    assert cfg.monitor.enabled is False
    assert cfg.data.seq_len == 256
    assert (cfg.optim.betas1, cfg.optim.betas2) == (0.8, 0.9)


def test_yaml_merge_left_to_right(tmp_path):
    a = tmp_path / "a.yaml"
    b = tmp_path / "b.yaml"
    a.write_text("optim:\n  lr: 0.1\n  weight_decay: 0.01\n")
    b.write_text("optim:\n  lr: 0.2\n")
    cfg = load_config(SFTConfig, [f"@{a}", f"@{b}"])
    assert cfg.optim.lr == 0.2 and cfg.optim.weight_decay == 0.01


def test_duplicate_yaml_keys_rejected(tmp_path):
    a = tmp_path / "dup.yaml"
    a.write_text("optim:\n  lr: 0.1\n  lr: 0.2\n")
    with pytest.raises(yaml.constructor.ConstructorError):
        load_yaml(a)


def test_help_lists_flags():
    h = help_text(SFTConfig)
    assert "--optim.lr" in h and "--data.seq-len" in h and "BOOL (also --no-...)" in h


def test_legacy_advantage_mode_normalised():
    cfg = RLConfig.model_validate({"orchestrator": {"advantage_mode": "group_reward", "normalize_group_advantages": True,
                                                    "length_penalty": "tokens"}})
    assert cfg.algo.type == "grpo" and cfg.algo.normalize_advantages is True
    assert cfg.algo.length_penalty.type == "tokens"


def test_legacy_sampling_and_loss_fields():
    cfg = RLConfig.model_validate({"inference": {"sampling": {"max_tokens": 64, "top_p": 0.9}},
                                   "loss": {"advantage_scale": 2.0}})
    assert cfg.inference.sampling.max_completion_tokens == 64
    assert cfg.loss.adv_tau == 2.0
    assert cfg.sampling_mask_required() is True


def test_rl_lora_capacity_rounding():
    cfg = RLConfig.model_validate({"lora": {"rank": 20}})
    assert cfg.inference.vllm.max_lora_rank == 32


def test_ckpt_validation():
    with pytest.raises(ValidationError):
        SFTConfig.model_validate({"ckpt": {"mode": "async"}})
    with pytest.raises(ValidationError):
        SFTConfig.model_validate({"ckpt": {"skip_optimizer": True}})
