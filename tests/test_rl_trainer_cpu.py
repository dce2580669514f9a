"""RL trainer step paths on CPU: streaming rollout chunks accumulate to the
same update as one whole batch, missing inference log-probs are recomputed
with the LoRA adapters disabled (and refused without adapters), context
parallelism over 2 gloo ranks matches the unsplit trainer, and the chunked
publisher's queue layout."""

import os
import random
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wavelet_b200.configs.config import RLConfig
from wavelet_b200.data.rl import RLExample


def _cfg(out, **extra):
    d = {
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 96, "fake_vocab_size": 64},
        "orchestrator": {"examples_per_step": 4, "rollouts_per_example": 2},
        "algo": {"type": "grpo"},
        "lora": None,
        "output_dir": str(out),
        "max_steps": 2,
        "optim": {"lr": 1e-2},
        "monitor": {"wandb": {"enabled": False}},
    }
    for k, v in extra.items():
        if isinstance(v, dict) and isinstance(d.get(k), dict):
            d[k] = {**d[k], **v}
        else:
            d[k] = v
    return RLConfig.model_validate(d)


def _examples(n=6, seed=0, with_ilp=True, vocab=64):
    rng = random.Random(seed)
    out = []
    for i in range(n):
        p = [rng.randrange(3, vocab) for _ in range(rng.randint(5, 12))]
        c = [rng.randrange(3, vocab) for _ in range(rng.randint(4, 20))]
        k = len(c)
        out.append(RLExample(prompt=[], completion=[], advantage=rng.uniform(-1, 1), reward=0.0,
                             input_ids=p + c, loss_mask=[False] * len(p) + [True] * k,
                             inference_logprobs=[rng.uniform(-4, -0.5) for _ in range(k)] if with_ilp else None,
                             temperatures=1.0))
    return out


def _trainer(out, **extra):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    from wavelet_b200.trainer.rl import RLTrainer

    return RLTrainer(_cfg(out, **extra)).setup()


@pytest.mark.parametrize("norm", ["token", "sequence"])
def test_streaming_chunks_match_whole_batch(tmp_path, norm):
    ex = _examples(7, seed=3)
    a = _trainer(tmp_path / "a", loss={"normalization": norm})
    b = _trainer(tmp_path / "b", loss={"normalization": norm})
    assert torch.equal(a.model.flat.compute, b.model.flat.compute)
    ma = a.train_on_examples(ex)
    mb = b.train_streaming_step(iter([ex[:3], ex[3:5], ex[5:]]))
    # the first AdamW moment is (1 - beta1) x the clipped gradient: compare
    # gradients there (the first Adam update is ~lr * sign(g), which flips for
    # near-zero gradients under any re-ordering of the sums)
    ga, gb = a.model.flat.exp_avg, b.model.flat.exp_avg
    torch.testing.assert_close(gb, ga, rtol=1e-3, atol=1e-6 * float(ga.abs().max()))
    assert abs(ma["loss"] - mb["loss"]) <= 1e-4 * max(1.0, abs(ma["loss"]))
    assert abs(ma["optim/grad_norm"] - mb["optim/grad_norm"]) <= 1e-3 * ma["optim/grad_norm"]
    assert ma["train/rl_units"] == mb["train/rl_units"]


def test_streaming_refuses_auxiliary_components(tmp_path):
    ex = _examples(4)
    for e in ex:
        e.ce_weight = 1.0
    t = _trainer(tmp_path)
    with pytest.raises(ValueError, match="non-streaming"):
        t.train_streaming_step(iter([ex[:2], ex[2:]]))


def test_missing_inference_logprobs_recomputed_with_adapters_disabled(tmp_path):
    from wavelet_b200.data.rl import make_rank_batches
    from wavelet_b200.ops import lm_head

    lora = {"rank": 4, "alpha": 8.0, "target_modules": ["q_proj", "v_proj", "down_proj"]}
    t = _trainer(tmp_path / "l", lora=lora)
    # make the adapters matter: non-zero B so the adapted and base models differ
    with torch.no_grad():
        t.model.lora.flat.compute.normal_(0.0, 0.05)
    ex = _examples(3, seed=5, with_ilp=False)
    (b,) = make_rank_batches(ex, 96, 0, 1, 1.0)
    assert bool(b.missing_inference().all() == b.loss_mask.all())
    m = t.model
    ctx = m.batch_ctx(b.base.position_ids, b.base.cu_seqlens, b.base.max_seqlen)
    t._recompute_inference_logprobs(b, ctx)
    with torch.no_grad(), m.adapters_disabled():
        h = m.hidden(b.base.input_ids, ctx)
        base_lp, _ = lm_head.ref.logprob_entropy(m.logits(h), b.base.targets.clamp_min(0), 1.0)
        h2 = m.hidden(b.base.input_ids, ctx)
    with torch.no_grad():
        lora_lp, _ = lm_head.ref.logprob_entropy(m.logits(m.hidden(b.base.input_ids, ctx)),
                                                 b.base.targets.clamp_min(0), 1.0)
    mk = b.loss_mask
    torch.testing.assert_close(b.inference_logprobs[mk], base_lp[mk].float(), rtol=1e-5, atol=1e-5)
    assert float((lora_lp[mk] - base_lp[mk]).abs().max()) > 1e-4  # the adapters were really off
    assert m.layers[0].lora is not None and m.lora is not None  # and are back on
    del h2
    met = t.train_on_examples(ex)  # the trainer path does the same inside the step
    assert torch.isfinite(torch.tensor(met["loss"]))
    plain = _trainer(tmp_path / "p")
    with pytest.raises(RuntimeError, match="no LoRA adapter"):
        plain.train_on_examples(_examples(2, with_ilp=False))


def _cp_worker(rank, world, init_file, out_dir, res):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.trainer.rl import RLTrainer

    t = RLTrainer(_cfg(out_dir, fsdp={"enabled": True, "impl": "fsdp2", "cp": world, "backend": "gloo"},
                       model={"attn_implementation": "sdpa"}, loss={"normalization": "token"})).setup()
    m = t.train_on_examples(_examples(5, seed=11))
    torch.save({"loss": m["loss"], "norm": m["optim/grad_norm"], "m1": t.model.flat.exp_avg.clone(),
                "shard": (t.model.flat.shard_slice.start, t.model.flat.shard_slice.stop)}, f"{res}.{rank}")
    dist.destroy_process_group()


def test_cp2_rl_step_matches_unsplit(tmp_path):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_cp_worker, args=(world, os.path.join(d, "init"), str(tmp_path / "cp"), os.path.join(d, "res")),
                 nprocs=world, join=True)
        got = [torch.load(os.path.join(d, f"res.{r}")) for r in range(world)]
    ref = _trainer(tmp_path / "ref", model={"attn_implementation": "sdpa"}, loss={"normalization": "token"})
    m = ref.train_on_examples(_examples(5, seed=11))
    full = ref.model.flat.exp_avg  # (1 - beta1) x the clipped gradient of the whole model
    for g in got:
        assert abs(g["loss"] - m["loss"]) <= 1e-4 * max(1.0, abs(m["loss"])), (g["loss"], m["loss"])
        assert abs(g["norm"] - m["optim/grad_norm"]) <= 2e-3 * m["optim/grad_norm"]
        sl = slice(*g["shard"])  # each cp rank owns a shard of the optimizer state over the dp x cp group
        n = g["m1"].numel()
        want = torch.nn.functional.pad(full, (0, max(0, sl.start + n - full.numel())))[sl.start:sl.start + n]
        torch.testing.assert_close(g["m1"], want, rtol=2e-3, atol=1e-6 * float(full.abs().max()))


def test_chunked_publisher_queue_layout(tmp_path):
    from wavelet_b200.orchestrator.async_scheduler import AsyncRolloutScheduler
    from wavelet_b200.transport.queue import (STABLE, FileSystemPolicyReceiver, FileSystemRolloutSender,
                                              stable_steps, step_dir)

    cfg = _cfg(tmp_path / "q", orchestrator={"examples_per_step": 5, "rollout_chunk_examples": 2,
                                             "max_async_level": 1}, policy_transfer={"poll_interval_seconds": 0.01})
    out = cfg.output_dir
    pd = step_dir(out / "policies", 0)
    pd.mkdir(parents=True)
    (pd / STABLE).touch()
    pd = step_dir(out / "policies", 1)
    pd.mkdir(parents=True)
    (pd / STABLE).touch()

    class Src:
        cursor = 0
        curriculum = None

        def take(self, n):
            self.cursor += n
            return list(range(self.cursor - n, self.cursor))

        def state_dict(self):
            return {"cursor": self.cursor}

    sizes = []

    class Orch:
        prompts = Src()
        engine = None

        def for_step(self, src):
            class V:
                last_stats = {}

                def materialize(self, step):
                    ids = src.take(99)[:0] if False else src.first
                    sizes.append((step, len(ids)))
                    return [RLExample([], [], 0.1, 1.0, input_ids=[i, i], loss_mask=[False, True]) for i in ids]

            return V()

    class Eng:
        def load_policy(self, d, *, step):
            pass

    sch = AsyncRolloutScheduler(cfg, Orch(), Eng(), FileSystemRolloutSender(out, cfg.transport),
                                FileSystemPolicyReceiver(out, cfg.policy_transfer))
    sch.run()
    q = out / "rollouts"
    assert stable_steps(q) == list(range(6))  # 3 chunks x 2 optimizer steps
    assert sorted(sizes) == [(0, 2), (1, 2), (2, 1), (3, 2), (4, 2), (5, 1)]
    mans = [sch.sender.stable_batch(s).manifest for s in range(6)]
    assert [(mm.optimizer_step, mm.chunk_index) for mm in mans] == [(0, 0), (0, 1), (0, 2), (1, 0), (1, 1), (1, 2)]

