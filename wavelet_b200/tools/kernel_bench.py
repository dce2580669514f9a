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


CASES = {"lm-head": lm_head, "decode-attention": decode_attention, "attention": attention, "gemm": gemm, "nf4-gemm": nf4_gemm,
         "generate": generate}


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
