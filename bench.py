#!/usr/bin/env python
"""Headline benchmark: SFT tokens/s on the Qwen2.5-7B-shaped dense model.

Contract (one JSON line from rank 0):
  python bench.py --gpus N --steps K --warmup W            (N=1)
  torchrun --nproc-per-node N bench.py --gpus N ...        (N>1, one rank per GPU)
  python bench.py --impl reference ...                     (reference arm)

Workload (the headline "Qwen2.5-7B-shaped dense SFT" configuration): 28 layers, hidden
3584, 28/4 heads x 128, SwiGLU 18944, vocab 152064 untied, RoPE 1e6, random
N(0, 0.02) init, bf16 compute / fp32 master + AdamW, sequences of 4096 uniform
random tokens with the loss masked on a random 10-40% prompt prefix.  Weak
scaling: every GPU runs 8 micro-batches of 1 x 4096 per optimizer step, so the
global batch is 8 x N sequences (64 at N = 8).  Data parallelism over N ranks
with sharded fp32 optimizer state and resident bf16 weights.

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
cuda.synchronize and CUDA events on the launching stream; the max over ranks is
reported.  The weights (15 GB) exceed the 126 MB L2, so no flush is needed.
A second timed run goes through the public ``SFTStepper.train_step`` API with
the micro-batches copied from pinned host memory each step and the loss read
back to the host (the "e2e" number).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

BASELINE_TOKS = None  # the reference publishes no number for this configuration


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--seq-len", type=int, default=None, help="default 4096 (sft) / 2048 (qlora)")
    p.add_argument("--micro-batches", type=int, default=None,
                   help="micro-batches of 1 sequence per GPU per step (default 8 for sft; 32/N for qlora)")
    p.add_argument("--layers", type=int, default=None, help="(debug only) override layer count; invalidates the number")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--workload", default="sft", choices=["sft", "qlora", "grpo-4b", "grpo-30b-a3b"],
                   help="sft: dense full fine-tune (headline); qlora: NF4 base + LoRA r16 on all projections; "
                        "grpo-4b: Qwen3-4B-shape GRPO step (native generator + trainer, integrated); "
                        "grpo-30b-a3b: Qwen3-30B-A3B-shape MoE GRPO step, expert parallel over all GPUs")
    p.add_argument("--activation-checkpointing", default="none", choices=["none", "full"],
                   help="none: keep every layer's activations (no recompute); full: recompute each layer in backward")
    p.add_argument("--tp", type=int, default=None,
                   help="tensor-parallel degree (default 1: data parallel over every GPU; 2 at 8 GPUs = dp4xtp2)")
    p.add_argument("--ref-attn", default="auto",
                   help="reference arm: model.attn_implementation (the reference's default 'auto' picks FA2 here)")
    p.add_argument("--comm", default="fabric", choices=["fabric", "nccl"],
                   help="optimizer-step collectives: fused peer-memory kernels (fabric) or NCCL")
    p.add_argument("--shard-params", action="store_true",
                   help="ZeRO-3: bf16 weights sharded over the data-parallel ranks, gathered layer by layer "
                        "(fsdp.shard_params); the optimizer collectives then run per layer over NCCL")
    return p.parse_args()


def reference_arm(args):
    """Runs the stock reference trainer from ``baseline/_ref`` (see
    ``baseline/reference_sft.py``); prints the same JSON line with
    ``"impl": "reference"``, or an ``unavailable`` line with the real reason."""
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "baseline"))
    rank = int(os.environ.get("RANK", "0"))
    if args.workload != "sft":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                f"reference arm for workload {args.workload!r} not run: the reference's RL path needs vLLM>=0.28 "
                "(image has 0.22) and its QLoRA path needs peft + bitsandbytes (neither installed)")}), flush=True)
        return 0
    try:
        import reference_sft
    except Exception as exc:  # the real error, not a canned reason
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"import failed: {type(exc).__name__}: {exc}"}),
                  flush=True)
        return 0
    return reference_sft.run(args, ClockSampler)


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sms.sort()
        med = sms[len(sms) // 2] if sms else None
        return {"sm_mhz": med, "sm_max_mhz": max(maxes) if maxes else None, "reasons": sorted(reasons), "samples": len(sms)}


RL_WORKLOADS = {
    # workload: (example config, model label, prompts per step, samples, prompt len, new tokens)
    "grpo-4b": ("examples/grpo_4b/rl.yaml", "Qwen3-4B-shape", 64, 8, 256, 1024),
    "grpo-30b-a3b": ("examples/grpo_30b_a3b/rl.yaml", "Qwen3-30B-A3B-shape (128 experts, top-8)", 32, 8, 512, 2048),
}


def rl_main(args):
    """GRPO step through the integrated RL runner (``wavelet rl`` with
    launcher.mode=integrated): every rank generates its share of the prompts x
    8 samples, scores and publishes them, then trains on the packed batch.
    grpo-4b: Qwen3-4B shape, data parallel; grpo-30b-a3b: Qwen3-30B-A3B shape
    with expert parallelism over all N ranks (expert dispatch / combine over
    peer memory) and a full generator replica per rank refreshed from the
    expert shards after every step.  Reports rollout tokens/s (generated
    tokens over device-timed generation, summed over ranks) and the
    device-timed step time (max over ranks)."""
    import tempfile

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.ops import _ext
    from wavelet_b200.orchestrator.runtime import IntegratedRunner
    from wavelet_b200.parallel.dist import destroy_distributed
    from wavelet_b200.utils.config import load_yaml

    root = os.path.dirname(os.path.abspath(__file__))
    cfg_path, label, prompts, samples, plen, new_tok = RL_WORKLOADS[args.workload]
    d = load_yaml(os.path.join(root, cfg_path))
    N = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    d["orchestrator"]["examples_per_step"] = max(1, prompts // N)
    if args.workload == "grpo-30b-a3b":
        d.setdefault("fsdp", {})["ep"] = N
        if N == 1:
            d["fsdp"]["enabled"] = False
    if args.layers:
        d["model"]["arch_overrides"] = {"num_layers": args.layers}
    d["output_dir"] = os.path.join(tempfile.gettempdir(), f"wavelet_b200_bench_rl_{os.environ.get('MASTER_PORT', 'x')}")
    d["clean_output_dir"] = True
    d["max_steps"] = args.warmup + args.steps
    cfg = RLConfig.model_validate(d)
    runner = IntegratedRunner(cfg).setup()
    _ext.load()
    dev = runner.world.device
    for _ in range(args.warmup):
        runner.run_step()
    sampler = ClockSampler(dev.index if dev.index is not None else 0) if rank == 0 else None
    if sampler:
        sampler.start()
    if N > 1:
        dist.barrier()
    torch.cuda.synchronize()
    gen_ms = step_ms = 0.0
    gen_tok = 0.0
    train_tok = 0.0
    with _ext.count_launches() as counter:
        for _ in range(args.steps):
            m = runner.run_step()
            gen_ms += m["time/generate_ms_device"]
            step_ms += m["time/step_ms_device"]
            gen_tok += m.get("rollout/generated_tokens", 0.0)
            train_tok += m.get("train/tokens", 0.0)
    torch.cuda.synchronize()
    if N > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    t = torch.tensor([gen_ms, step_ms, gen_tok, train_tok], device=dev, dtype=torch.float64)
    if N > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm)
        gen_ms, step_ms, gen_tok, train_tok = mx[0].item(), mx[1].item(), sm[2].item(), sm[3].item()
    else:
        gen_ms, step_ms, gen_tok, train_tok = t.tolist()
    K = args.steps
    value = gen_tok / (gen_ms / 1000.0)
    if rank == 0:
        par = (f"integrated ep{N} (experts sharded over every rank; dense weights data parallel; "
               "each rank generates on a full replica)" if args.workload == "grpo-30b-a3b"
               else f"integrated dp{N} (each rank generates and trains)")
        rec = {
            "metric": f"RL rollout tok/s ({label} GRPO, native generator)",
            "value": value, "unit": "tokens/s", "n_gpus": N, "steps": K, "warmup": args.warmup,
            "ms_per_step": step_ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16",
            "data": f"synthetic (uniform random {plen}-token prompts, reversed-prompt reward, random-init weights)",
            "config": {"model": label + (f" ({args.layers} layers: INVALID debug run)" if args.layers else ""),
                       "prompts_per_step": prompts, "samples_per_prompt": samples,
                       "prompt_len": plen, "max_new_tokens": new_tok, "temperature": 1.0,
                       "parallelism": par,
                       "l2": "inputs larger than L2 (8 GB of weights, tens of GB of KV per step)"},
            "rl_step_ms": step_ms / K, "generate_ms_per_step": gen_ms / K,
            "train_tokens_per_step": train_tok / K, "generated_tokens_per_step": gen_tok / K,
            "gpu_launches": counter.count, "clocks": clocks,
            "e2e": {"value": value, "unit": "tokens/s",
                    "h2d_bytes_per_step": int(train_tok / K * 32), "d2h_bytes_per_step": int(gen_tok / K * 12),
                    "note": "the RL step is end to end by construction: rollouts return to the host (token ids and "
                            "log-probs), pass through the filesystem queue and are copied back for training"},
        }
        print(json.dumps(rec), flush=True)
    destroy_distributed()
    return 0


def optimizer_parity_check(engine, groups, dp, tp, hyper, lr, dev) -> dict:
    """One optimizer step of the fused peer-memory kernels checked against an
    NCCL + fp32 PyTorch oracle on the same gradients (run once, untimed).

    Before the fused step: NCCL ``reduce_scatter_tensor`` of the same fp32
    gradient buffer (the oracle shard), the oracle global norm from it, and
    copies of a window of this rank's fp32 master / moments.  After it: the
    fused reduce-scatter output against the oracle shard (whole shard), the
    fused grad norm against the oracle norm, the fused AdamW master window
    against a plain fp32 AdamW of the oracle gradient, and the bf16 parameters
    that every peer stored into this rank's replica (the fused all-gather)
    against the peers' master windows gathered over NCCL.  Returns the max
    over ranks of each error."""
    import torch
    import torch.distributed as dist

    from wavelet_b200.parallel.zero import FusedShardedAdamW

    opt = engine.opt
    assert isinstance(opt, FusedShardedAdamW)
    flat = engine.model.trainable
    n = flat.shard_numel
    g_ref = torch.empty(n, device=dev, dtype=torch.float32)
    dist.reduce_scatter_tensor(g_ref, flat.grad, op=dist.ReduceOp.SUM, group=groups.dp)
    st = torch.zeros(2, device=dev, dtype=torch.float32)
    opt.local_sumsq_(g_ref, st)
    st64 = st.double()
    dist.all_reduce(st64)  # world: every dp x tp rank
    norm_ref = float(st64[0]) ** 0.5
    factor = min(1.0, hyper.max_grad_norm / (norm_ref + 1e-6)) if hyper.max_grad_norm > 0 else 1.0
    wlen = min(n, 1 << 22)
    win = slice(n - wlen, n)  # the tail of the shard: matrices (TP-sharded region under TP)
    p0, m0, v0 = flat.master[win].clone(), flat.exp_avg[win].clone(), flat.exp_avg_sq[win].clone()
    step = opt.step_count + 1
    out = opt.step(lr)
    g_err = (opt.g_shard - g_ref).abs().max() / g_ref.abs().max().clamp_min(1e-30)
    # fp32 AdamW oracle on the window, fed the fused reduce-scatter output and
    # clip factor (the reduce-scatter and the norm are checked against NCCL above)
    b1, b2 = hyper.betas
    g = opt.g_shard[win] * out["clip_factor"]
    m1 = b1 * m0 + (1 - b1) * g
    v1 = b2 * v0 + (1 - b2) * g * g
    p1 = p0 * (1 - lr * hyper.weight_decay) - (lr / (1 - b1 ** step)) * m1 / (
        v1.sqrt() / (1 - b2 ** step) ** 0.5 + hyper.eps)
    p_err = (flat.master[win] - p1).abs().max()
    # fused all-gather: every peer's window as stored into this rank's bf16 replica
    mine16 = flat.master[win].to(torch.bfloat16)
    allw = torch.empty(dp * wlen, device=dev, dtype=torch.bfloat16)
    dist.all_gather_into_tensor(allw, mine16, group=groups.dp)
    comp = flat.compute.detach()
    ag_bad = torch.zeros((), device=dev, dtype=torch.float32)
    for r in range(dp):
        lo = r * n + (n - wlen)
        ag_bad += (comp[lo:lo + wlen] != allw[r * wlen:(r + 1) * wlen]).sum().float()
    res = torch.stack([g_err.float(), p_err.float(), ag_bad,
                       torch.tensor(abs(out["grad_norm"] - norm_ref) / max(norm_ref, 1e-30), device=dev)])
    dist.all_reduce(res, op=dist.ReduceOp.MAX)
    res = res.tolist()
    return {"rs_grad_max_rel_err": res[0], "adamw_master_max_abs_err": res[1], "allgather_mismatches": int(res[2]),
            "grad_norm_rel_err": res[3], "grad_norm": norm_ref, "clip_factor_oracle": factor,
            "window_elems_per_rank": wlen,
            "oracle": "NCCL reduce_scatter + NCCL all_reduce(norm) + fp32 torch AdamW + NCCL all_gather",
            "ok": bool(res[0] <= 1e-5 and res[1] <= 1e-6 and res[2] == 0 and res[3] <= 1e-4)}


def main():
    args = parse()
    if args.tp is None:
        # data parallel at every N by default: the reference's tensor-parallel
        # path (Hugging Face tp_plan) needs `accelerate`, which this image lacks,
        # so dp is the layout both arms run; --tp 2 runs dp(N/2) x tp2 here
        args.tp = 1
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload in RL_WORKLOADS:
        return rl_main(args)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from wavelet_b200.models.config import resolve_arch
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.ops import _ext
    from wavelet_b200.parallel.dist import Groups, ParallelDims, destroy_distributed, init_distributed
    from wavelet_b200.parallel.fabric import Fabric, maybe_fabric
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.data.fake import synthetic_sft_microbatches
    from wavelet_b200.trainer.engine import Engine
    from wavelet_b200.trainer.sft_step import SFTStepper

    world = init_distributed(timeout_s=900)
    rank, N = world.rank, world.world_size
    assert N == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={N}"
    dev = world.device
    _ext.load()
    qlora = args.workload == "qlora"
    tp = args.tp
    if N % tp:
        raise SystemExit(f"--tp {tp} must divide --gpus {N}")
    if qlora and tp > 1:
        raise SystemExit("the QLoRA workload runs data-parallel only (--tp 1)")
    dims = ParallelDims(tp=tp, world_size=N)
    groups = Groups(dims, rank)
    dp, dp_rank = dims.dp, groups.dp_rank

    overrides = {"num_layers": args.layers} if args.layers else None
    cfg = resolve_arch(args.model, overrides)
    zero3 = args.shard_params
    if zero3 and (qlora or tp > 1):
        raise SystemExit("--shard-params runs the dense workload data-parallel only")
    fabric = maybe_fabric(dp, dp_rank, dev, group=groups.dp) if (args.comm == "fabric" and not zero3) else None
    norm_fabric = Fabric(rank, N, dev) if (fabric is not None and tp > 1) else None
    tp_fabric = Fabric(groups.tp_rank, tp, dev, group=groups.tp) if (tp > 1 and args.comm == "fabric") else None
    lora = None
    if qlora:
        from types import SimpleNamespace

        lora = SimpleNamespace(rank=16, alpha=32.0, dropout=0.0, target_modules=[
            "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"])
    model = build_model(cfg, dev, torch.bfloat16, dp_rank=dp_rank, dp_world=dp, seed=1234, fabric=fabric,
                        lora=lora, load_in_4bit=qlora, tp=(tp, groups.tp_rank) if tp > 1 else None,
                        shard_params=zero3)
    if zero3:
        from wavelet_b200.parallel.zero3 import ParamGatherer

        ParamGatherer(model, group=groups.dp if dp > 1 else None)
    model.tp_group = groups.tp
    if tp_fabric is not None:
        model.attach_tp_fabric(tp_fabric)
    hyper = AdamWHyper(lr=2e-4 if qlora else 1e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                       max_grad_norm=1.0)
    model.set_activation_checkpointing(1 if args.activation_checkpointing == "full" else None)
    engine = Engine(model, hyper, dp_group=groups.dp, dp_world=dp, fabric=fabric, norm_fabric=norm_fabric)
    stepper = SFTStepper(engine, dev)

    S = args.seq_len or (2048 if qlora else 4096)
    # micro-batches of one sequence per data-parallel rank and step: the global
    # batch is 8 sequences per GPU at every layout (64 at 8 GPUs)
    mb = args.micro_batches or (max(1, 32 // N) if qlora else 8 * tp)
    # distinct batches every step (TP peers share their data-parallel rank's data)
    n_dev = args.warmup + args.steps
    n_host = 0 if args.no_e2e else args.steps
    sets = [synthetic_sft_microbatches(mb, S, cfg.vocab_size, seed=100003 * i + 101 * dp_rank + 7)
            for i in range(n_dev + n_host)]
    dev_sets = [[b.to(dev) for b in st] for st in sets[:n_dev]]
    host_sets = [[b.pin_memory() for b in st] for st in sets[n_dev:]]
    torch.cuda.synchronize()
    it = iter(range(n_dev))

    def step_device():
        return stepper.train_step(dev_sets[next(it)], hyper.lr, device_resident=True)

    for _ in range(args.warmup):
        step_device()

    parity = None
    if N > 1 and fabric is not None and not qlora:
        # one extra, untimed step on a warm-up batch: fused collectives vs the NCCL oracle
        scale = 1.0 / engine.global_token_count(float(dev_sets[0][0].loss_mask.sum()), dev)
        engine.sft_micro_step(dev_sets[0][0], scale)
        model.finalize_grads()
        parity = optimizer_parity_check(engine, groups, dp, tp, hyper, hyper.lr, dev)
        torch.cuda.synchronize()

    sampler = ClockSampler(dev.index if dev.index is not None else 0) if rank == 0 else None
    if sampler:
        sampler.start()
    if N > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with _ext.count_launches() as counter:
        start.record()
        for _ in range(args.steps):
            out = step_device()
        end.record()
    torch.cuda.synchronize()
    if N > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_local = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms_local], device=dev, dtype=torch.float64)
    if N > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    launches = counter.count
    tokens_per_step = dp * mb * S
    value = tokens_per_step / (ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        stepper.h2d_bytes = stepper.d2h_bytes = 0
        if N > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e_s = torch.cuda.Event(enable_timing=True)
        e_e = torch.cuda.Event(enable_timing=True)
        e_s.record()
        for i in range(args.steps):
            stepper.train_step(host_sets[i], hyper.lr)
        e_e.record()
        torch.cuda.synchronize()
        te = torch.tensor([e_s.elapsed_time(e_e) / args.steps], device=dev, dtype=torch.float64)
        if N > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {
            "value": tokens_per_step / (float(te.item()) / 1000.0),
            "unit": "tokens/s",
            "h2d_bytes_per_step": stepper.h2d_bytes // args.steps,
            "d2h_bytes_per_step": stepper.d2h_bytes // args.steps,
            "ms_per_step": float(te.item()),
        }

    from wavelet_b200.trainer.perf import flops_per_token

    mfu_flops = flops_per_token(cfg, S, model.lora.num_trainable() if model.lora is not None else None)
    layout = f"dp{dp}" + (f"xtp{tp}" if tp > 1 else "") + ("-zero3" if zero3 else "")
    if rank == 0:
        rec = {
            "metric": ("QLoRA SFT tok/s (Qwen2.5-7B-shape, NF4 base, LoRA r16 all projections)" if qlora
                       else "SFT tok/s (Qwen2.5-7B-shape dense SFT, bf16)"),
            "value": value,
            "unit": "tokens/s",
            "n_gpus": N,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong" if qlora else "weak",
            "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None,
            "dtype": "bf16",
            "data": "synthetic (uniform random tokens, a new batch every step, random-init weights)",
            "config": {
                "model": "Qwen2.5-7B-shape" + (f" ({args.layers} layers: INVALID debug run)" if args.layers else ""),
                "global_batch": dp * mb,
                "seq_len": S,
                "micro_batch": 1,
                "grad_accum": mb,
                "parallelism": layout,
                **({"base": "NF4 blocksize 64 (fp32 absmax), frozen", "lora": "r=16 alpha=32 on q/k/v/o/gate/up/down"}
                   if qlora else {}),
                "optimizer": "AdamW (fp32 master, sharded)" + (" on LoRA adapters" if qlora else ""),
                "activation_checkpointing": args.activation_checkpointing,
                "optimizer_comm": ("fused peer-memory RS+AdamW+AG kernels" if fabric is not None
                                   else ("per-layer NCCL weight gathers and gradient reductions (ZeRO-3)" if zero3
                                         else ("NCCL reduce-scatter/all-gather" if dp > 1
                                               else "none (1 data-parallel rank)"))),
                **({"tp_comm": "fused GEMM->all-reduce epilogue over peer memory" if tp_fabric is not None
                    else "NCCL all-reduce"} if tp > 1 else {}),
                "l2": "inputs larger than L2 (15 GB of weights read per micro-step)",
            },
            "mfu": value * mfu_flops / (N * 2.25e15),
            "loss": out["loss"],
            "gpu_launches": launches,
            "clocks": clocks,
            "e2e": e2e,
            **({"fused_vs_nccl": parity} if parity is not None else {}),
        }
        print(json.dumps(rec), flush=True)
    for fab in (fabric, norm_fabric, tp_fabric):
        if fab is not None:
            fab.close()
    destroy_distributed()
    return 0


if __name__ == "__main__":
    sys.exit(main())
