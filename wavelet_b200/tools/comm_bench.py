"""``torchrun --nproc-per-node N -m wavelet_b200.tools.comm_bench``: the fused
compute + collective paths of one NVLink node against their NCCL baselines.

Every case is timed on the device (CUDA events on the launching stream, 3
warm-up calls, ``--iters`` timed calls bracketed by a barrier and a
synchronize), the time is the max over ranks, and rank 0 prints one JSON
line per case with the achieved fraction of the roofline: the slower of the
math at the measured GEMM peak, the local HBM bytes at the measured copy
bandwidth and the bytes this rank must move over NVLink at the measured peer
copy bandwidth (770 GB/s per direction).

Cases:
  tp-ar    row-parallel GEMM + all-reduce (7B o_proj / down_proj shapes):
           fused peer-store GEMM + slot sum vs the same GEMM + NCCL all-reduce
  optim    ZeRO optimizer step over a flat store: fused RS + norm + AdamW + AG
           kernels vs NCCL reduce-scatter / all-reduce / all-gather around the
           same AdamW kernel
  ep       MoE token exchange (30B-A3B shape, top-8 of 128 experts): dispatch
           + combine over peer memory vs NCCL all-to-all (transfers only)
  refresh  expert policy refresh: pull-gather of every rank's expert shard
           into the full tensor vs NCCL all-gather
  policy   split-placement policy transfer (--model shape): the first half of
           the ranks are trainer replicas, the second half generators; the
           peer push of every trainer rank's share into every generator's
           receive slot vs an NCCL broadcast of the flat buffer from trainer
           rank 0 (the reference's transport), plus the generator's slot load
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _peaks() -> tuple[float, float]:
    p = Path("MEASURED_PEAKS.json")
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    return 1590.0, 6650.0


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def _roof(flops: float = 0.0, hbm: float = 0.0, nvl: float = 0.0) -> float:
    tf, gbs = _peaks()
    return max(flops / (tf * 1e9), hbm / (gbs * 1e6), nvl / (NVLINK_GBS * 1e6))  # ms


def tp_ar(a, fab, rank, world) -> list[dict]:
    from .. import ops
    from ..parallel.tp_fabric import TPFabric

    out = []
    tpf = TPFabric(fab, capacity=1 << 22)
    for name, N, Kfull in (("o_proj", 3584, 3584), ("down_proj", 3584, 18944)):
        M, K = a.tokens, Kfull // world
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        res = torch.randn(M, N, device="cuda").bfloat16()

        def nccl():
            y = ops.gemm(x, w, res=res if rank == 0 else None)
            dist.all_reduce(y)

        fused_ms = _time(lambda: tpf.gemm_allreduce(x, w, res=res), a.iters)
        nccl_ms = _time(nccl, a.iters)
        gemm_ms = _time(lambda: ops.gemm(x, w), a.iters)
        flops = 2.0 * M * N * K
        roof = _roof(flops=flops, nvl=(world - 1) * M * N * 2)
        out.append({"case": "tp-ar", "layer": name, "M": M, "N": N, "K": K, "world": world,
                    "fused_ms": fused_ms, "gemm_nccl_ms": nccl_ms, "gemm_only_ms": gemm_ms,
                    "speedup_vs_nccl": nccl_ms / fused_ms, "roofline_ms": roof, "frac_of_roofline": roof / fused_ms})
    return out


def optim(a, fab, rank, world) -> list[dict]:
    from ..models.params import FlatParams, ParamSpec
    from ..parallel.zero import AdamWHyper, FusedShardedAdamW, ShardedAdamW

    n = a.params
    specs = [ParamSpec("w", (n,))]
    h = AdamWHyper(lr=1e-4)
    fl_f = FlatParams(specs, "cuda", torch.bfloat16, rank, world, alloc=fab.allocator())
    fl_n = FlatParams(specs, "cuda", torch.bfloat16, rank, world)
    for fl in (fl_f, fl_n):
        fl.init_(seed=1)
        fl.grad.normal_(0, 1e-3)
    fused, ref = FusedShardedAdamW(fl_f, h, fab), ShardedAdamW(fl_n, h, dist.group.WORLD, world)

    # the step zeroes the gradients; the kernels do the same work on zeros
    fused_ms = _time(lambda: fused.step(check_finite=False), a.iters)
    nccl_ms = _time(lambda: ref.step(check_finite=False), a.iters)
    N = fl_f.numel
    shard = N // world
    nvl = (world - 1) * shard * 4 + (world - 1) * shard * 2  # pull fp32 grad shards, push bf16 params
    hbm = N * 4 + shard * (4 * 2 + 8 * 2) + N * 2  # grads read, master + moments r/w, params written
    roof = _roof(hbm=hbm, nvl=nvl)
    return [{"case": "optim", "params": N, "world": world, "fused_ms": fused_ms, "nccl_ms": nccl_ms,
             "speedup_vs_nccl": nccl_ms / fused_ms, "roofline_ms": roof, "frac_of_roofline": roof / fused_ms}]


def ep(a, fab, rank, world) -> list[dict]:
    from ..parallel.ep_fabric import FabricEP

    T, H, E, k = a.tokens, 2048, 128, 8
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    topi = torch.rand(T, E, device="cuda", generator=g).argsort(1)[:, :k].contiguous()  # k distinct experts
    x = torch.randn(T, H, device="cuda").bfloat16()
    fe = FabricEP(fab, dist.group.WORLD, E, H, capacity=T * k * 2)
    p = fe.plan(topi)
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    w = torch.full((T, k), 1.0 / k, device="cuda")

    def fused():
        fe.dispatch("xs", x, p)
        fe.view("y", p.R).copy_(fe.view("xs", p.R))  # stands in for the expert GEMMs
        fe.combine("y", p, k, w, x, out)

    # NCCL baseline: copies sorted by destination rank, variable-split all-to-all both ways
    dst = (topi.reshape(-1) // (E // world))
    order = torch.argsort(dst, stable=True)
    send_counts = torch.bincount(dst, minlength=world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    src_tok = torch.arange(T, device="cuda").repeat_interleave(k)[order]
    recv = torch.empty(sum(rc), H, device="cuda", dtype=torch.bfloat16)
    back = torch.empty(T * k, H, device="cuda", dtype=torch.bfloat16)

    def nccl():
        send = x.index_select(0, src_tok)
        dist.all_to_all_single(recv, send, rc, sc)
        y = recv.clone()
        dist.all_to_all_single(back, y, sc, rc)
        o = x.float().index_add_(0, src_tok, back.float() * (1.0 / k))
        return o

    fused_ms = _time(fused, a.iters)
    nccl_ms = _time(nccl, a.iters)
    remote = sum(c for r, c in enumerate(sc) if r != rank)
    nvl = remote * H * 2  # per direction: this rank's remote copies out (dispatch) and back (combine)
    roof = 2 * _roof(nvl=nvl)
    return [{"case": "ep", "tokens": T, "H": H, "experts": E, "top_k": k, "world": world, "fused_ms": fused_ms,
             "nccl_ms": nccl_ms, "speedup_vs_nccl": nccl_ms / fused_ms, "roofline_ms": roof,
             "frac_of_roofline": roof / fused_ms}]


def refresh(a, fab, rank, world) -> list[dict]:
    from .. import ops

    n = a.params // world // 8 * 8
    buf = fab.alloc(n, torch.bfloat16)
    buf.tensor.normal_()
    full = torch.empty(n * world, device="cuda", dtype=torch.bfloat16)
    m = ops.ext()

    def fused():
        fab.barrier()
        m.gather_from_peers(buf.ptrs, world, 0, n, full)
        fab.barrier()

    fused_ms = _time(fused, a.iters)
    nccl_ms = _time(lambda: dist.all_gather_into_tensor(full, buf.tensor), a.iters)
    roof = _roof(hbm=n * world * 2 * 2, nvl=(world - 1) * n * 2)
    return [{"case": "refresh", "shard_params": n, "world": world, "fused_ms": fused_ms, "nccl_ms": nccl_ms,
             "speedup_vs_nccl": nccl_ms / fused_ms, "roofline_ms": roof, "frac_of_roofline": roof / fused_ms}]


def policy(a, fab, rank, world) -> list[dict]:
    import tempfile

    from ..models.config import resolve_arch
    from ..models.qwen import build_model
    from ..transport.peer_policy import PeerPolicyReceiver, PeerPolicySender, used_numel

    if world < 2 or world % 2:
        raise ValueError("the policy case needs an even world size (trainers + generators)")
    T = world // 2
    trainer = rank < T
    tgroup = dist.new_group(list(range(T)))
    bgroup = dist.new_group([0] + list(range(T, world)))  # NCCL baseline: trainer rank 0 + generators
    m = build_model(resolve_arch(a.model), torch.device("cuda", torch.cuda.current_device()), torch.bfloat16,
                    seed=0 if trainer else 1, with_grad=False, with_optimizer=False)
    n = used_numel(m.flat)
    root = [tempfile.mkdtemp(prefix="wb_policy_bench_") if rank == 0 else None]
    dist.broadcast_object_list(root, src=0)
    rec = None if trainer else PeerPolicyReceiver(m, root[0], rank - T, slots=2)
    dist.barrier()
    snd = (PeerPolicySender(m, root[0], rank=rank, world=T, expect=world - T, timeout_s=60,
                            barrier=lambda: dist.barrier(group=tgroup)) if trainer else None)
    kern, proto = [], []
    for step in range(3 + a.iters):
        dist.barrier()
        if trainer:
            info = snd.push(step)
            if step >= 3:
                kern.append(info["kernel_ms"])
                proto.append(1e3 * info["push_seconds"])
    dist.barrier()
    load_ms = 0.0
    if not trainer:
        rec.load(2 + a.iters, timeout_s=60)
    # every generator now holds trainer rank 0's weights: compare per-parameter sums
    sums = torch.stack([m.flat.view(nm).float().sum() for nm in m.flat.names()])
    every = [torch.empty_like(sums) for _ in range(world)]
    dist.all_gather(every, sums)
    match = all(torch.equal(every[0], every[g]) for g in range(T, world))
    if not trainer:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            m.flat.compute.copy_(rec.bufs[0])
        e1.record()
        torch.cuda.synchronize()
        load_ms = e0.elapsed_time(e1) / a.iters
    stats = torch.tensor([sum(kern) / len(kern) if kern else 0.0, sum(proto) / len(proto) if proto else 0.0,
                          load_ms], device="cuda")
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    buf = m.flat.compute[:n]

    def bcast():
        if rank == 0 or not trainer:
            dist.broadcast(buf, src=0, group=bgroup)

    nccl_ms = _time(bcast, a.iters)
    if snd is not None:
        snd.close()
    dist.barrier()
    if rec is not None:
        rec.close()
    G = world - T
    nbytes = n * 2
    roof = _roof(nvl=nbytes * max(G / T, 1.0))  # a generator's ingress, or a trainer rank's egress
    return [{"case": "policy", "model": a.model, "bytes": nbytes, "trainers": T, "generators": G,
             "push_kernel_ms": float(stats[0]), "push_protocol_ms": float(stats[1]), "nccl_broadcast_ms": nccl_ms,
             "generator_load_ms": float(stats[2]), "weights_match": match, "roofline_ms": roof, "frac_of_roofline": roof / float(stats[0]),
             "speedup_vs_nccl": nccl_ms / float(stats[0])}]


CASES = {"tp-ar": tp_ar, "optim": optim, "ep": ep, "refresh": refresh, "policy": policy}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--cases", default="tp-ar,optim,ep,refresh")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--params", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--model", default="qwen3-4b", help="architecture of the policy case")
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    from ..parallel.fabric import Fabric

    fab = Fabric(rank, world, dev)
    try:
        for c in a.cases.split(","):
            for row in CASES[c](a, fab, rank, world):
                if rank == 0:
                    print(json.dumps(row), flush=True)
        fab.check()
    finally:
        fab.close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
