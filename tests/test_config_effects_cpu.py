"""Settings from the reference's schema either act or are named: inert keys
set away from their default are listed with the reason; keys this framework
implements take effect (do_sample, max_prompt_tokens, num_generations,
enforce_eager / cuda_graphs, the LM-head chunk, skip_scheduler, the state
server's event bound, the tokenizer's chat template); unsupported values are
refused (repetition_penalty, lora.modules_to_save, generator TP)."""

import pytest

from wavelet_b200.configs.config import RLConfig, SFTConfig
from wavelet_b200.configs.inert import inert_settings


def test_inert_keys_are_named_with_reasons():
    cfg = RLConfig.model_validate({"inference": {"vllm": {"quantization": "fp8", "enable_fp32_lm_head": False,
                                                          "gpu_memory_utilization": 0.5}},
                                   "model": {"compile": True}, "policy_transfer": {"nccl_dtype": "float32"}})
    msgs = inert_settings(cfg)
    keys = {m.split("=")[0] for m in msgs}
    assert keys == {"inference.vllm.quantization", "inference.vllm.enable_fp32_lm_head", "model.compile",
                    "policy_transfer.nccl_dtype"}
    assert all("has no effect here" in m for m in msgs)
    assert inert_settings(RLConfig()) == [] and inert_settings(SFTConfig()) == []
    # set to its default value: not a change, not named
    assert inert_settings(RLConfig.model_validate({"model": {"compile": False}})) == []
    sft = SFTConfig.model_validate({"data": {"num_workers": 4}, "loss_impl": "liger"})
    assert {m.split("=")[0] for m in inert_settings(sft)} == {"loss_impl"}  # num_workers prefetches in SFT
    rl = RLConfig.model_validate({"data": {"num_workers": 1}})
    assert {m.split("=")[0] for m in inert_settings(rl)} == {"data.num_workers"}


def test_unsupported_values_are_refused():
    with pytest.raises(ValueError, match="repetition_penalty"):
        RLConfig.model_validate({"inference": {"sampling": {"repetition_penalty": 1.1}}})
    with pytest.raises(ValueError, match="modules_to_save"):
        SFTConfig.model_validate({"lora": {"modules_to_save": ["embed_tokens"]}})


def test_sampling_keys_act(tmp_path, monkeypatch):
    import torch

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    from wavelet_b200.inference.policy import NativePolicyInferenceEngine
    from wavelet_b200.orchestrator.rollouts import PromptRecord, RLOrchestrator

    cfg = RLConfig.model_validate({"model": {"name": "tiny", "random_init": True},
                                   "inference": {"sampling": {"do_sample": False, "num_generations": 3,
                                                              "max_prompt_tokens": 4, "temperature": 0.7}},
                                   "orchestrator": {"rollouts_per_example": 2}, "output_dir": str(tmp_path)})
    eng = NativePolicyInferenceEngine(cfg)
    p = eng.sampling()
    assert p.temperature == 0.0 and p.n == 3
    orch = RLOrchestrator(cfg, engine=None, sender=None, prompts=None)
    assert orch._sampling().temperature == 0.0

    seen = []

    class Eng:
        def generate(self, prompts, params):
            seen.extend(prompts)
            raise RuntimeError("stop")

    orch.engine = Eng()
    with pytest.raises(RuntimeError, match="stop"):
        orch.generate_records([PromptRecord(list(range(10)), example_id="a")], 0)
    assert seen == [[6, 7, 8, 9]]  # the last max_prompt_tokens tokens
    with pytest.raises(NotImplementedError, match="torchrun group"):
        NativePolicyInferenceEngine(RLConfig.model_validate({"inference": {"vllm": {"tensor_parallel_size": 2}}})).setup()


def test_generator_graphs_lm_head_chunk_and_state_events():
    from types import SimpleNamespace

    from wavelet_b200.inference.hf_generator import make_generator
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.ops.lm_head import DEFAULT_CHUNK
    from wavelet_b200.orchestrator.state_server import OrchestratorRunState
    from wavelet_b200.trainer.model_options import lm_head_chunk

    import torch

    g = make_generator(build_model(PRESETS["tiny"], "cpu", torch.float32, seed=0), max_num_seqs=4,
                       max_model_len=64, cuda_graphs=False)
    assert g.use_graphs is False
    assert lm_head_chunk(SimpleNamespace(fused_lm_head_token_chunk_size=1024)) == 1024
    assert lm_head_chunk(SimpleNamespace(fused_lm_head_token_chunk_size="disabled")) == DEFAULT_CHUNK
    st = OrchestratorRunState("/tmp", max_events=100)
    for i in range(150):
        st.event("e", i=i)
    assert len(st.events()) == 100


def test_chat_template_overrides_the_tokenizer(tmp_path):
    from wavelet_b200.data.tokenizer import load_tokenizer

    with pytest.raises(ValueError, match="chat_template"):
        load_tokenizer("tiny", chat_template="{{ messages }}")


def test_rollout_columns_round_trip_under_renames():
    from wavelet_b200.configs.config import RLDataConfig
    from wavelet_b200.data.rl import RLExample, example_from_payload, example_to_payload

    e = RLExample(prompt=[], completion=[], advantage=0.5, reward=1.0, input_ids=[1, 2, 3],
                  loss_mask=[False, True, True], inference_logprobs=[-0.1, -0.2], temperatures=0.7)
    plain = example_to_payload(e, RLDataConfig())
    assert "advantage" in plain and "temperatures" in plain  # default names: the on-disk format is unchanged
    data = RLDataConfig.model_validate({"advantage_column": "adv", "inference_logprobs_column": "lp"})
    row = example_to_payload(e, data)
    assert "adv" in row and "lp" in row and "advantage" not in row
    back = example_from_payload(row, data)
    assert back.advantage == 0.5 and back.inference_logprobs == [-0.1, -0.2]
    # an external file written with custom column names
    ext = {"input_ids": [1, 2], "loss_mask": [False, True], "adv": -1.0, "reward": 0.0, "prompt": [], "completion": []}
    assert example_from_payload(ext, data).advantage == -1.0


def test_rollout_selection_is_checked():
    with pytest.raises(ValueError, match="requires examples_per_step"):
        RLConfig.model_validate({"orchestrator": {"batch_selection": "rollouts", "refill_zero_advantage": False}})
    with pytest.raises(ValueError, match="refill_zero_advantage=false"):
        RLConfig.model_validate({"orchestrator": {"batch_selection": "rollouts", "examples_per_step": 2}})
    RLConfig.model_validate({"orchestrator": {"batch_selection": "rollouts", "examples_per_step": 2,
                                              "refill_zero_advantage": False}})
    msgs = inert_settings(RLConfig.model_validate({"orchestrator": {"max_pending_rollout_chunks": 2}}))
    assert msgs and msgs[0].startswith("orchestrator.max_pending_rollout_chunks")


def test_sample_rows_ratio_cap_and_decoding():
    from types import SimpleNamespace

    from wavelet_b200.data.rl import RLExample
    from wavelet_b200.data.tokenizer import CharTokenizer
    from wavelet_b200.trainer.rl import sample_rows

    recs = [RLExample(prompt=[], completion=[], advantage=0.1 * i, reward=float(i), input_ids=[70, 71, 72 + i],
                      loss_mask=[False, False, True], metadata={"example_id": f"e{i}"}) for i in range(20)]
    sc = SimpleNamespace(sample_ratio=0.25, max_samples=3)
    rows = sample_rows(recs, sc, seed=1, step=4)
    assert len(rows) == 3 and rows == sample_rows(recs, sc, seed=1, step=4)
    assert rows[0]["prompt_ids"] == [70, 71] and rows[0]["completion_tokens"] == 1
    assert len(sample_rows(recs, SimpleNamespace(sample_ratio=0.25, max_samples=None), 1, 4)) == 5
    assert sample_rows(recs, SimpleNamespace(sample_ratio=0.0, max_samples=None), 1, 4) == []
    dec = sample_rows(recs[:1], SimpleNamespace(sample_ratio=None, max_samples=None), 1, 4, CharTokenizer())
    assert isinstance(dec[0]["completion"], str) and dec[0]["example_id"] == "e0"


def test_per_environment_sampling_group_size_and_algorithm(tmp_path):
    """orchestrator.envs[] entries: group_size and sampling apply to that
    environment's prompts only; an entry's algorithm scores its records;
    data_path reaches the loader; a per-environment curriculum is refused."""
    import json as _json

    from wavelet_b200.inference.engine import Completion
    from wavelet_b200.orchestrator.rollouts import PromptRecord, RLOrchestrator

    rows = tmp_path / "eq.jsonl"
    rows.write_text("".join(_json.dumps({"question": f"q{i}", "answer": str(i)}) + "\n" for i in range(4)))
    from wavelet_b200.configs.config import VERIFIER_ROLLOUT_FUNCTION

    vf = {"custom_rollout_function": VERIFIER_ROLLOUT_FUNCTION}
    with pytest.raises(ValueError, match="curriculum"):
        RLConfig.model_validate({"launcher": {"mode": "process"}, "orchestrator": {
            **vf, "max_async_level": 1, "envs": [{"id": "equation_builder", "curriculum": {}}]}})
    cfg = RLConfig.model_validate({"launcher": {"mode": "process"},
                                   "orchestrator": {**vf, "rollouts_per_example": 2, "max_async_level": 1, "envs": [
                                       {"id": "equation_builder", "group_size": 3, "sampling": {"temperature": 0.3},
                                        "algo": {"type": "reward"}}]}})
    orch = RLOrchestrator(cfg, engine=None, sender=None, prompts=None)
    name = next(iter(orch.env_cfg))
    calls = []

    class Eng:
        def generate(self, prompts, params):
            calls.append((len(prompts), params.n, params.temperature))
            return [Completion(i, j, p, [1, 2], [-0.1, -0.2], "length") for i, p in enumerate(prompts)
                    for j in range(params.n)]

    orch.engine = Eng()
    ps = [PromptRecord([5, 6], metadata={"env": name}), PromptRecord([7], metadata={"env": "other"}),
          PromptRecord([8, 9], metadata={"env": name})]
    recs = orch.generate_records(ps, 0)
    assert sorted(calls) == sorted([(2, 3, 0.3), (1, 2, 1.0)])
    assert sum(1 for r in recs if r.metadata["env"] == name) == 6 and all(
        r.temperatures == 0.3 for r in recs if r.metadata["env"] == name)
    from dataclasses import replace

    scored = orch.score([replace(r, reward=0.5) for r in recs])
    assert len(scored) == len(recs)
    from types import SimpleNamespace

    from wavelet_b200.orchestrator.runtime import env_args

    assert env_args(SimpleNamespace(args={"k": 1}, data_path=rows)) == {"k": 1, "path": str(rows)}


def test_sft_prefetching_dataset_keeps_the_consumed_state():
    from wavelet_b200.data.sft import PrefetchingDataset, SFTDataset

    cfg = SFTConfig.model_validate({"data": {"source": "fake", "seq_len": 64, "fake_vocab_size": 50,
                                             "num_workers": 2}}).data
    plain = SFTDataset(cfg, None, seed=3)
    want = [plain.next_micro_batch().input_ids.tolist() for _ in range(4)]
    ds = SFTDataset(cfg, None, seed=3)
    pre = PrefetchingDataset(ds, 4)
    got = [pre.next_micro_batch().input_ids.tolist() for _ in range(2)]
    assert got == want[:2]
    import time

    time.sleep(0.2)  # the producer runs ahead ...
    st = pre.state_dict()  # ... but the state is the one after the second batch the trainer took
    fresh = SFTDataset(cfg, None, seed=3)
    fresh.load_state_dict(st)
    assert fresh.next_micro_batch().input_ids.tolist() == want[2]
    assert len(pre.samples()) == len(plain.samples())  # the wrapped dataset's other methods
    pre.close()
