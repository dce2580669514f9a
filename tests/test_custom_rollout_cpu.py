"""User rollout functions (orchestrator.custom_rollout_function = "module:function",
ref orchestrator/rollouts.py:263-275, 510-525): the function gets the step's
prompt records and returns scored rollouts; advantages are assigned per group."""

from __future__ import annotations

import pytest

from wavelet_b200.configs.config import RLConfig

MODULE = '''
from dataclasses import replace

CALLS = []


def rollout(orchestrator, records, engine):
    CALLS.append((orchestrator, len(records), engine))
    out = []
    for r in records:
        p = r.metadata["prompt_ids"]
        for k in range(2):
            out.append(replace(r, input_ids=p + [5, 6], loss_mask=[False] * len(p) + [True, True],
                               inference_logprobs=[-0.1, -0.2], reward=float(k)))
    return out


def unscored(orchestrator, records, engine):
    return records


not_callable = 3
'''


def _cfg(tmp_path, fn):
    return RLConfig.model_validate({
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 64, "fake_vocab_size": 64, "fake_prompt_len": 4},
        "orchestrator": {"custom_rollout_function": fn, "examples_per_step": 3, "rollouts_per_example": 2},
        "reward": {"mode": "reverse_match"}, "algo": {"type": "grpo"},
        "lora": None, "output_dir": str(tmp_path / "out")})


@pytest.fixture
def user_module(tmp_path, monkeypatch):
    (tmp_path / "my_rollouts.py").write_text(MODULE)
    monkeypatch.syspath_prepend(str(tmp_path))
    import importlib
    import sys

    sys.modules.pop("my_rollouts", None)
    return importlib.import_module("my_rollouts")


def _orch(cfg, engine="ENGINE"):
    from wavelet_b200.orchestrator.rollouts import RLOrchestrator
    from wavelet_b200.orchestrator.runtime import build_prompt_source

    return RLOrchestrator(cfg, engine, None, build_prompt_source(cfg, 64))


def test_user_rollout_function_replaces_generation(tmp_path, user_module):
    orch = _orch(_cfg(tmp_path, "my_rollouts:rollout"))
    recs = orch.materialize(1)
    who, n, engine = user_module.CALLS[-1]
    assert who is orch and n == 3 and engine == "ENGINE"
    assert len(recs) == 6
    # the function's rewards are kept (the configured reverse_match reward is not applied)
    assert sorted(r.reward for r in recs) == [0.0, 0.0, 0.0, 1.0, 1.0, 1.0]
    groups = {}
    for r in recs:
        groups.setdefault(r.metadata["group"], []).append(r.advantage)
    assert len(groups) == 3 and all(abs(sum(a)) < 1e-6 and len(a) == 2 for a in groups.values())
    assert orch.last_stats["rollout/custom_records"] == 6.0


def test_user_rollout_function_errors(tmp_path, user_module):
    with pytest.raises(ValueError, match="without a reward"):
        _orch(_cfg(tmp_path, "my_rollouts:unscored")).materialize(0)
    with pytest.raises(TypeError, match="not callable"):
        _orch(_cfg(tmp_path, "my_rollouts:not_callable"))
    with pytest.raises(ValueError, match="module.path:function_name"):
        _orch(_cfg(tmp_path, "my_rollouts.rollout"))


def test_reference_verifiers_function_name_selects_verifiers():
    from wavelet_b200.configs.config import RLOrchestratorConfig

    for name in ("wavelet.orchestrator.verifiers:generate_rollouts", "verifiers"):
        assert RLOrchestratorConfig(custom_rollout_function=name).uses_verifiers
    assert not RLOrchestratorConfig(custom_rollout_function="my_rollouts:rollout").uses_verifiers
