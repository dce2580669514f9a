"""``python -m wavelet_b200.tools.kernel_bench``: CUDA-event timings of the
framework's kernels on synthetic inputs (3 warm-up calls, then the mean of
``--iters`` timed calls bracketed by synchronisation), printed as one JSON
line per case with achieved bandwidth or FLOP rate.  The same commands are
what the profile summaries capture under ``ncu``.

Cases:
  decode-attention  paged GQA decode attention over head-major KV pages
  attention         varlen causal attention forward + backward
  gemm              dense tcgen05 GEMM (forward / dgrad / wgrad layouts)
  nf4-gemm          NF4-B GEMM (in-kernel dequantisation, small M)
  lm-head           chunked LM-head cross-entropy forward + backward (logit
                    GEMM, softmax stats, in-place dL/dz, dgrad and fp32 wgrad)
  generate          the native generator end to end (prefill + decode)
  router            MoE router (softmax, top-k, renormalised weights, expert
                    counts) against the same in torch
  sampling          top-k / top-p thresholds + Gumbel sampling of a decode
                    batch against torch topk / sort / multinomial
  adamw8            8-bit-moment AdamW and fp32 AdamW flat kernels against
                    torch's fused AdamW over the same elements
  policy-push       reshard + cast push of a policy (local destination)
                    against torch copies of the same segments
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import time

import torch


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters  # ms


def decode_attention(a) -> dict:
    from .. import ops

    B, ctx, Hq, Hk, bs = a.batch, a.ctx, a.heads, a.kv_heads, 64
    nb = -(-(ctx + 1) // bs)
    kc = torch.randn(B * nb + 1, Hk, bs, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.arange(B * nb, dtype=torch.int32, device="cuda").view(B, nb)
    cl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, 128, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    ms = _time(lambda: ops.ext().decode_attention(q, kc, vc, bt, cl, out, a.splits, 1 / math.sqrt(128)), a.iters)
    byt = B * ctx * Hk * 128 * 2 * 2
    return {"case": "decode-attention", "batch": B, "ctx": ctx, "Hq": Hq, "Hk": Hk, "splits": a.splits,
            "us": ms * 1e3, "GB/s": byt / ms / 1e6}


def attention(a) -> dict:
    from ..ops.attention import attention_bwd, attention_fwd

    S, n, Hq, Hk = a.ctx, a.batch, a.heads, a.kv_heads
    T = S * n
    q = torch.randn(T, Hq, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, Hk, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, Hk, 128, device="cuda", dtype=torch.bfloat16)
    cu = torch.arange(0, T + 1, S, device="cuda", dtype=torch.int32)
    o, lse = attention_fwd(q, k, v, cu, S, True)
    do = torch.randn_like(o)
    fl = 4 * n * S * S * Hq * 128 / 2
    tf = _time(lambda: attention_fwd(q, k, v, cu, S, True), a.iters)
    tb = _time(lambda: attention_bwd(do, q, k, v, o, lse, cu, S, True), a.iters)
    return {"case": "attention", "seq": S, "seqs": n, "Hq": Hq, "Hk": Hk, "fwd_ms": tf, "fwd_TFLOPs": fl / tf / 1e9,
            "bwd_ms": tb, "bwd_TFLOPs": 2.5 * fl / tb / 1e9}


def gemm(a) -> dict:
    from .. import ops

    M, N, K = a.m, a.n, a.k
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    g = torch.zeros(N, K, device="cuda", dtype=torch.float32)
    fl = 2 * M * N * K
    out = {"case": "gemm", "M": M, "N": N, "K": K}
    out["fwd_TFLOPs"] = fl / _time(lambda: ops.gemm(x, w), a.iters) / 1e9
    out["dgrad_TFLOPs"] = fl / _time(lambda: ops.gemm(dy, w, b_mn=True), a.iters) / 1e9
    out["wgrad_TFLOPs"] = fl / _time(lambda: ops.gemm(dy, x, a_mn=True, b_mn=True, out=g, epi=ops.EPI_F32_ACC),
                                     a.iters) / 1e9
    return out


def nf4_gemm(a) -> dict:
    from .. import ops
    from ..ops.nf4 import quantize

    M, N, K = a.m, a.n, a.k
    q = quantize(torch.randn(N, K, device="cuda") * 0.02)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ops.gemm(x, q), a.iters)
    return {"case": "nf4-gemm", "M": M, "N": N, "K": K, "us": ms * 1e3, "TFLOPs": 2 * M * N * K / ms / 1e9,
            "weight_GB/s": q.nbytes() / ms / 1e6}


def generate(a) -> dict:
    from ..inference.engine import Generator, SamplingParams
    from ..models.config import resolve_arch
    from ..models.qwen import build_model

    cfg = resolve_arch(a.model)
    m = build_model(cfg, "cuda", torch.bfloat16, seed=1, with_grad=False, with_optimizer=False)
    gen = Generator(m, max_num_seqs=max(512, a.batch * a.samples), max_model_len=a.ctx + a.new_tokens + 64,
                    gpu_memory_utilization=0.5)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (a.ctx,), generator=g).tolist() for _ in range(a.batch)]
    gen.generate(prompts[:2], SamplingParams(max_tokens=8, n=a.samples, seed=0))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = gen.generate(prompts, SamplingParams(temperature=1.0, max_tokens=a.new_tokens, n=a.samples, seed=1))
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    n = sum(len(c.token_ids) for c in out)
    return {"case": "generate", "model": a.model, "prompts": a.batch, "samples": a.samples, "prompt_len": a.ctx,
            "new_tokens": a.new_tokens, "seconds": dt, "tokens/s": n / dt, **gen.stats}


def lm_head(a) -> dict:
    """Whole-vocabulary CE of ``--m`` tokens (hidden ``--k``, vocabulary
    ``--n``): three GEMMs of 2*T*H*V FLOPs plus two row passes over the bf16
    logit chunk; the [T, V] logits are never held whole."""
    from ..ops import lm_head as lmh

    T, H, V = a.m, a.k, a.n
    h = (torch.randn(T, H, device="cuda") * 0.5).bfloat16()
    W = (torch.randn(V, H, device="cuda") * 0.02).bfloat16()
    gW = torch.zeros(V, H, device="cuda")
    tgt = torch.randint(0, V, (T,), device="cuda")
    wts = torch.full((T,), 1.0 / T, device="cuda")
    ms = _time(lambda: lmh.sft_loss_and_grad(h, W, tgt, wts, gW, chunk=a.chunk), a.iters)
    flops = 3 * 2.0 * T * H * V
    return {"case": "lm-head", "tokens": T, "hidden": H, "vocab": V, "chunk": a.chunk, "ms": ms,
            "tflops": flops / (ms * 1e9)}


def router(a) -> dict:
    """``--m`` tokens routed over ``--n`` experts, top ``--k``."""
    from .. import ops

    T, E, k = a.m, a.n, a.k
    logits = torch.randn(T, E, device="cuda")
    probs = torch.empty(T, E, device="cuda")
    topi = torch.empty(T, k, device="cuda", dtype=torch.int64)
    topv = torch.empty(T, k, device="cuda")
    w = torch.empty(T, k, device="cuda")
    ssum = torch.empty(T, device="cuda")
    counts = torch.zeros(E, device="cuda", dtype=torch.int32)

    def ours():
        counts.zero_()
        ops.ext().moe_route(logits, k, True, True, probs, topi, topv, w, ssum, counts)

    def torch_ref():
        p = torch.softmax(logits.bfloat16().float(), -1)
        v, i = torch.topk(p, k, -1)
        s_ = v.sum(-1, keepdim=True)
        return v / s_, i, torch.bincount(i.reshape(-1), minlength=E)

    ms, ms_t = _time(ours, a.iters), _time(torch_ref, a.iters)
    v_t, i_t, c_t = torch_ref()
    ours()
    # bf16 logits tie often; the kernel breaks ties towards the lower index and
    # torch.topk in no fixed order: compare the selected probability values
    same = bool(torch.allclose(topv.sort(-1).values, torch.softmax(logits.bfloat16().float(), -1)
                               .gather(1, i_t).sort(-1).values, rtol=1e-5, atol=1e-7))
    return {"case": "router", "tokens": T, "experts": E, "top_k": k, "us": ms * 1e3, "torch_us": ms_t * 1e3,
            "speedup_vs_torch": ms_t / ms, "same_as_torch": same}


def sampling(a) -> dict:
    """A decode step's sampling: ``--batch`` rows of ``--n`` logits, top-k
    ``--k`` and top-p 0.9 at temperature 1."""
    from .. import ops
    from ..inference.engine import sampling_thresholds_reference

    B, V, K = a.batch, a.n, a.k
    z = (torch.randn(B, V, device="cuda") * 3).bfloat16()
    inv = torch.ones(B, device="cuda")
    tk = torch.full((B,), K, device="cuda", dtype=torch.int32)
    tp = torch.full((B,), 0.9, device="cuda")
    th = torch.empty(B, device="cuda")
    tok = torch.empty(B, device="cuda", dtype=torch.long)
    lp = torch.empty(B, device="cuda")
    rows = torch.arange(B, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(0)

    def ours():
        ops.ext().sample_thresholds(z, tk, tp, inv, th)
        ops.ext().sample_tokens(z, inv, th, 0.0, 7, rows, tok, lp, None)

    def torch_ref():  # thresholds with topk / sort, then masked softmax + multinomial
        zf = z.float()
        kth = torch.topk(zf, K, -1).values[:, -1:]
        srt = torch.sort(zf, -1, descending=True).values
        cum = torch.softmax(srt, -1).cumsum(-1)
        idx = (cum < 0.9).sum(-1, keepdim=True).clamp_max(V - 1)
        pth = srt.gather(1, idx)
        keep = zf >= torch.maximum(kth, pth)
        p = torch.softmax(zf.masked_fill(~keep, float("-inf")), -1)
        t = torch.multinomial(p, 1, generator=gen)
        return t, torch.log(p.gather(1, t))

    ms, ms_t = _time(ours, a.iters), _time(torch_ref, a.iters)
    ours()
    ref = sampling_thresholds_reference(z[:4], [K] * 4, [0.9] * 4, inv[:4])
    return {"case": "sampling", "rows": B, "vocab": V, "top_k": K, "top_p": 0.9, "us": ms * 1e3,
            "torch_us": ms_t * 1e3, "speedup_vs_torch": ms_t / ms,
            "thresholds_match_reference": bool(torch.equal(th[:4], ref.to(th.device)))}


def adamw8(a) -> dict:
    """``--m`` x 2^20 parameters: fp32 master + bf16 shadow, two moments."""
    from .. import ops

    n = a.m << 20
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda") * 1e-3
    p16 = p.bfloat16()
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    nb = (n + ops.Q8_BLOCK - 1) // ops.Q8_BLOCK
    m8, v8 = torch.zeros(n, device="cuda", dtype=torch.int8), torch.zeros(n, device="cuda", dtype=torch.uint8)
    am, av = torch.zeros(nb, device="cuda"), torch.zeros(nb, device="cuda")
    kw = dict(lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, step=3)
    ms8 = _time(lambda: ops.adamw8_flat_(p, g, m8, v8, am, av, p16, **kw), a.iters)
    ms32 = _time(lambda: ops.adamw_flat_(p, g, m, v, p16, **kw), a.iters)
    tp = torch.nn.Parameter(p.clone())
    tp.grad = g.clone()
    opt = torch.optim.AdamW([tp], lr=1e-4, weight_decay=0.01, fused=True)
    ms_t = _time(opt.step, a.iters)
    # bytes moved: p (rw fp32), g (r fp32), p16 (w), moments (rw) — 8-bit codes + block scales vs fp32
    b8 = n * (4 * 2 + 4 + 2 + 1 * 4) + nb * 4 * 4
    b32 = n * (4 * 2 + 4 + 2 + 4 * 4)
    return {"case": "adamw8", "params": n, "adamw8_ms": ms8, "adamw_fp32_ms": ms32, "torch_fused_adamw_ms": ms_t,
            "adamw8_GB/s": b8 / ms8 / 1e6, "adamw_fp32_GB/s": b32 / ms32 / 1e6,
            "state_bytes_per_param": {"adamw8": 4 + 2 + 2 * 4 / ops.Q8_BLOCK, "fp32": 12}}


def policy_push(a) -> dict:
    """Push a ``--model`` policy from one flat store into another of the same
    layout on this GPU (each parameter a segment), bf16 -> bf16."""
    from .. import ops
    from ..models.config import resolve_arch
    from ..models.qwen import build_model
    from ..transport.peer_policy import push_segments

    m = build_model(resolve_arch(a.model), "cuda", torch.bfloat16, seed=0, with_grad=False, with_optimizer=False)
    dst = torch.empty_like(m.flat.compute)
    segs = push_segments(m, dict(m.flat.offsets))["flat"]
    table = torch.tensor(segs, dtype=torch.int64)
    ms = _time(lambda: ops.ext().policy_push(m.flat.compute, [dst.data_ptr()], dst.numel(), True, table), a.iters)
    views = [(m.flat.compute[s[0]:s[0] + s[3]], dst[s[1]:s[1] + s[3]]) for s in segs]

    def torch_ref():
        for src, d in views:
            d.copy_(src)

    ms_t = _time(torch_ref, a.iters)
    nbytes = sum(s[2] * s[3] for s in segs) * 2
    return {"case": "policy-push", "model": a.model, "bytes": nbytes, "segments": len(segs), "ms": ms,
            "GB/s (read+write)": 2 * nbytes / ms / 1e6, "torch_copies_ms": ms_t, "speedup_vs_torch": ms_t / ms}


CASES = {"lm-head": lm_head, "decode-attention": decode_attention, "attention": attention, "gemm": gemm, "nf4-gemm": nf4_gemm,
         "generate": generate, "router": router, "sampling": sampling, "adamw8": adamw8, "policy-push": policy_push}


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="python -m wavelet_b200.tools.kernel_bench", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("case", choices=sorted(CASES))
    p.add_argument("--batch", type=int, default=128, help="sequences / prompts")
    p.add_argument("--ctx", type=int, default=1024, help="context / sequence / prompt length")
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--splits", type=int, default=1)
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--model", default="qwen3-4b")
    p.add_argument("--samples", type=int, default=8)
    p.add_argument("--new-tokens", type=int, default=256)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--chunk", type=int, default=4096, help="lm-head token chunk")
    a = p.parse_args(sys.argv[1:] if argv is None else argv)
    from ..ops import _ext

    _ext.load()
    print(json.dumps(CASES[a.case](a)), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
