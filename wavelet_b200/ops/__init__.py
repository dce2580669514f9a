"""Fused operators of wavelet_b200.

Every op has two implementations selected by the device of its inputs:

* CUDA tensors run the hand-written sm_100a kernels of the in-tree ``wb_C``
  extension (``wavelet_b200/csrc``).  There is no silent fallback: if the
  extension cannot be loaded on a GPU machine the op raises.
* CPU tensors run the float32 PyTorch formulation in ``ops.reference`` (the
  CPU/gloo plumbing configuration and the numerics oracle).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import reference as ref
from ._ext import load as _load_ext

EPI_BF16 = 0
EPI_F32 = 1
EPI_F32_ACC = 2


def ext():
    """The loaded CUDA extension (raises if it cannot be built/loaded)."""
    return _load_ext()


# --------------------------------------------------------------------- GEMM
def gemm(a: torch.Tensor, b, *, a_mn: bool = False, b_mn: bool = False,
         out: Optional[torch.Tensor] = None, epi: int = EPI_BF16, alpha: float = 1.0,
         bias: Optional[torch.Tensor] = None, res: Optional[torch.Tensor] = None,
         a2: Optional[torch.Tensor] = None, b2: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C[M, N] = alpha * (A(m, k) B(n, k) + A2(m, j) B2(n, j)) (+ bias + res) on the tcgen05 GEMM.

    ``a`` is [M, K] (K-major) or [K, M] with ``a_mn``; ``b`` is [N, K] or [K, N]
    with ``b_mn``, or an ``NF4Weight`` (dequantised inside the kernel).
    ``a2``/``b2`` (same majorness as ``a``/``b``) add a second product into the
    same accumulator (the LoRA-fused linear).  ``epi`` selects bf16 store,
    fp32 store or fp32 accumulate.
    """
    from .nf4 import FUSED_MAX_M, NF4Weight, dequant_cache, nf4_table

    quant = isinstance(b, NF4Weight)
    M = a.shape[1] if a_mn else a.shape[0]
    if quant:
        N = b.cols if b_mn else b.rows
    else:
        N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        if epi == EPI_BF16:
            dtype = torch.bfloat16 if a.is_cuda else a.dtype
        else:
            dtype = torch.float32
        out = torch.empty(M, N, device=a.device, dtype=dtype)
    if not a.is_cuda:
        A = a.t() if a_mn else a
        Bm = b.dequantize(torch.float32) if quant else b
        B = Bm if b_mn else Bm.t()
        r = A.float() @ B.float()
        if a2 is not None:
            A2 = a2.t() if a_mn else a2
            B2 = b2 if b_mn else b2.t()
            r = r + A2.float() @ B2.float()
        r = alpha * r
        if bias is not None:
            r = r + bias.float()
        if res is not None:
            r = r + res.float()
        if epi == EPI_F32_ACC:
            out.add_(r)
        else:
            out.copy_(r)
        return out
    if not quant and a2 is None:
        S = _splitk(M, N, a.shape[0] if a_mn else a.shape[1], a_mn, epi, out)
        if S > 1:
            return _gemm_splitk(a, b, b_mn, out, S, alpha, bias, res)
        ext().gemm(a, a_mn, b, b_mn, out, epi, alpha, bias, res)
        return out
    if quant and M > FUSED_MAX_M:
        # training-size M: dequantise once (cached), then the dense GEMM
        b = dequant_cache().get(b)
        quant = False
        if a2 is None:
            ext().gemm(a, a_mn, b, b_mn, out, epi, alpha, bias, res)
            return out
    if quant:
        ext().gemm_ex(a, a_mn, None, b_mn, out, N, epi, alpha, bias, res, a2, b2, b.codes, b.absmax, b.rows,
                      b.cols, list(nf4_table()))
    else:
        ext().gemm_ex(a, a_mn, b, b_mn, out, N, epi, alpha, bias, res, a2, b2, None, None, 0, 0, [0.0] * 16)
    return out


def gemm_grouped(a, a_mn, b, b_mn, c, mode, M, N, K, tile_group=None, b_group_stride=0, b_outer=0, k_start=None,
                 k_len=None, groups=0, epi=EPI_BF16, alpha=1.0):
    """Grouped (MoE expert) GEMM; see ``csrc/gemm.h``.  CPU: a per-group loop."""
    if a.is_cuda:
        ext().gemm_grouped(a, a_mn, b, b_mn, c, mode, M, N, K, tile_group, b_group_stride, b_outer, k_start, k_len,
                           groups, epi, alpha)
        return c
    if mode == 1:  # rows of A in 128-row tiles, tile t uses weight block tile_group[t]
        for t, g in enumerate(tile_group.tolist()):
            r0, r1 = t * 128, min(M, (t + 1) * 128)
            Bg = b[g * b_group_stride : g * b_group_stride + (K if b_mn else N)]
            B = Bg if b_mn else Bg.t()
            r = alpha * (a[r0:r1].float() @ B.float())
            c[r0:r1] = r.to(c.dtype) if epi == EPI_BF16 else (c[r0:r1] + r if epi == EPI_F32_ACC else r)
        return c
    for g in range(groups):  # mode 2: C[g] (op)= A_g^T B_g over token rows
        k0, kl = int(k_start[g]), int(k_len[g])
        if kl == 0:
            continue
        r = alpha * (a[k0 : k0 + kl].float().t() @ b[k0 : k0 + kl].float())
        blk = c[g * M : (g + 1) * M]
        if epi == EPI_F32_ACC:
            blk.add_(r)
        else:
            blk.copy_(r)
    return c


_SMS = 148
_KRANGES: dict = {}


def _splitk(M: int, N: int, K: int, a_mn: bool, epi: int, out) -> int:
    """Split K when a bf16-output GEMM has too few 128x256 tiles to fill the
    SMs (skinny generation GEMMs); every split keeps >= 8 k-blocks."""
    if a_mn or epi != EPI_BF16 or M > 2048 or N % 4 or (out.stride(0) % 4):
        return 1
    tiles = -(-M // 128) * -(-N // 256)
    if tiles * 2 > _SMS:
        return 1
    s = min(8, _SMS // tiles, K // 512)  # tiles * s <= one wave of CTAs
    return s if s > 1 else 1


def _gemm_splitk(a, b, b_mn, out, S, alpha, bias, res):
    M, K = a.shape
    N = out.shape[1]
    kb = -(-K // 64)
    per = -(-kb // S)
    S = -(-kb // per)  # every range non-empty (an empty one would leave its partial unwritten)
    key = (a.device, K, S)
    kr = _KRANGES.get(key)
    if kr is None:
        starts = [min(K, i * per * 64) for i in range(S)]
        lens = [max(0, min(K, (i + 1) * per * 64) - starts[i]) for i in range(S)]
        kr = (torch.tensor(starts, dtype=torch.int32, device=a.device),
              torch.tensor(lens, dtype=torch.int32, device=a.device))
        _KRANGES[key] = kr
    ws = torch.empty(S * M, N, device=a.device, dtype=torch.float32)
    ext().gemm_grouped(a, False, b, b_mn, ws, 2, M, N, K, None, 0, 0, kr[0], kr[1], S, EPI_F32, 1.0)
    ext().splitk_reduce(ws, S, out, bias, res, alpha)
    return out


class LinearFn(torch.autograd.Function):
    """y = x W^T (+ b); the weight gradient is accumulated in fp32 directly
    into ``main_grad`` by the GEMM epilogue (no bf16 dW is materialised)."""

    @staticmethod
    def forward(ctx, x, w, b, main_grad, bias_grad):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        y = gemm(x2, w, bias=b)
        ctx.save_for_backward(x2, w)
        ctx.main_grad = main_grad
        ctx.bias_grad = bias_grad
        ctx.has_bias = b is not None
        ctx.shp = shp
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, w.shape[0]).contiguous()
        dx = gemm(dy2, w, b_mn=True)
        dw = None
        if ctx.main_grad is not None:
            gemm(dy2, x2, a_mn=True, b_mn=True, out=ctx.main_grad, epi=EPI_F32_ACC)
        elif ctx.needs_input_grad[1]:
            dw = gemm(dy2, x2, a_mn=True, b_mn=True, epi=EPI_F32).to(w.dtype)
        db = None
        if ctx.has_bias:
            s = dy2.float().sum(0)
            if ctx.bias_grad is not None:
                ctx.bias_grad.add_(s)
            else:
                db = s.to(w.dtype)
        return dx.view(ctx.shp), dw, db, None, None


def linear(x, w, b=None, main_grad=None, bias_grad=None):
    if not x.is_cuda:
        return torch.nn.functional.linear(x, w, b)
    return LinearFn.apply(x, w, b, main_grad, bias_grad)


# ------------------------------------------------------------------ RMSNorm
def rmsnorm_fwd(x, w, eps, res=None, want_h=False):
    """Returns (y, rstd, h) with h = x + res when ``res`` is given."""
    x = x.contiguous()
    if not x.is_cuda:
        h = x + res if res is not None else x
        hf = h.float()
        rstd = torch.rsqrt(hf.pow(2).mean(-1) + eps)
        y = (hf * rstd[..., None] * w.float()).to(x.dtype)
        return y, rstd, h
    y = torch.empty_like(x)
    rows = x.numel() // x.shape[-1]
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    h = torch.empty_like(x) if (res is not None and want_h) else None
    ext().rmsnorm_fwd(x, res, h, w, y, rstd, eps)
    return y, rstd, h


def rmsnorm_bwd(x, w, rstd, dy, dres=None, dw=None):
    if not x.is_cuda:
        xf, wf, dyf = x.float(), w.float(), dy.float()
        xh = xf * rstd[..., None]
        g = dyf * wf
        dx = rstd[..., None] * (g - xh * (g * xh).mean(-1, keepdim=True))
        if dres is not None:
            dx = dx + dres.float()
        if dw is not None:
            dw.add_((dyf * xh).reshape(-1, x.shape[-1]).sum(0).to(dw.dtype))
        return dx.to(x.dtype)
    dx = torch.empty_like(x)
    ext().rmsnorm_bwd(x, w, rstd, dy.contiguous(), dres, dx, dw)
    return dx


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, w_grad):
        y, rstd, _ = rmsnorm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        ctx.w_grad = w_grad
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        if ctx.w_grad is not None:
            dx = rmsnorm_bwd(x, w, rstd, dy, dw=ctx.w_grad)
            return dx, None, None, None
        dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        dx = rmsnorm_bwd(x, w, rstd, dy, dw=dw)
        return dx, dw.to(w.dtype), None, None


def rmsnorm(x, w, eps=1e-6, w_grad=None):
    if not x.is_cuda:
        return ref.rmsnorm(x, w, eps)
    return RMSNormFn.apply(x, w, eps, w_grad)


# ----------------------------------------------------------------- SwiGLU
def swiglu_fwd(gu):
    if not gu.is_cuda:
        return ref.swiglu(gu)
    I = gu.shape[-1] // 2
    h = torch.empty(*gu.shape[:-1], I, device=gu.device, dtype=gu.dtype)
    ext().swiglu_fwd(gu.contiguous(), h)
    return h


def swiglu_bwd(gu, dh):
    if not gu.is_cuda:
        I = gu.shape[-1] // 2
        g, u = gu[..., :I].float(), gu[..., I:].float()
        sg = torch.sigmoid(g)
        d = dh.float()
        return torch.cat([d * u * sg * (1 + g * (1 - sg)), d * g * sg], -1).to(gu.dtype)
    dgu = torch.empty_like(gu)
    ext().swiglu_bwd(gu.contiguous(), dh.contiguous(), dgu)
    return dgu


# ----------------------------------------------------------- QK-norm + RoPE
def qk_norm_rope_(qkv, n_q, n_k, pos, inv_freq, q_w=None, k_w=None, eps=1e-6):
    """In place on the q and k heads of a packed [T, (n_q+2 n_k) * 128] qkv row."""
    if not qkv.is_cuda:
        T = qkv.shape[0]
        hd = 2 * inv_freq.numel()
        heads = qkv[:, : (n_q + n_k) * hd].view(T, n_q + n_k, hd)
        x = heads
        if q_w is not None:
            q = ref.rmsnorm(x[:, :n_q], q_w, eps)
            k = ref.rmsnorm(x[:, n_q:], k_w, eps)
            x = torch.cat([q, k], 1)
        heads.copy_(ref.apply_rope(x, pos, inv_freq))
        return None
    rstd = torch.empty(qkv.shape[0] * (n_q + n_k), device=qkv.device, dtype=torch.float32) if q_w is not None else None
    ext().qk_norm_rope_fwd(qkv, n_q, n_k, pos, inv_freq, q_w, k_w, rstd, eps)
    return rstd


# ---------------------------------------------------------------- embedding
def embedding_fwd(table, ids):
    if not table.is_cuda:
        return table[ids]
    out = torch.empty(ids.numel(), table.shape[1], device=table.device, dtype=table.dtype)
    ext().embedding_fwd(table, ids.reshape(-1).contiguous(), out)
    return out


def embedding_bwd_(dy, ids, dtable):
    if not dy.is_cuda:
        dtable.index_add_(0, ids.reshape(-1), dy.to(dtable.dtype))
        return
    ext().embedding_bwd(dy.contiguous(), ids.reshape(-1).contiguous(), dtable)


def qk_norm_rope_bwd_(dqkv, qkv_pre, n_q, n_k, pos, inv_freq, q_w, k_w, rstd, dq_w, dk_w, eps=1e-6):
    """In place: d(qkv) through RoPE (and the per-head QK RMSNorm); weight
    gradients accumulate into ``dq_w`` / ``dk_w``.  CPU: autograd through the
    reference forward."""
    if dqkv.is_cuda:
        ext().qk_norm_rope_bwd(dqkv, qkv_pre, n_q, n_k, pos, inv_freq, q_w, k_w, rstd, dq_w, dk_w)
        return
    T = qkv_pre.shape[0]
    hd = 2 * inv_freq.numel()
    with torch.enable_grad():
        x = qkv_pre[:, : (n_q + n_k) * hd].view(T, n_q + n_k, hd).detach().float().requires_grad_(True)
        leaves = [x]
        y = x
        if q_w is not None:
            qw = q_w.detach().float().requires_grad_(True)
            kw = k_w.detach().float().requires_grad_(True)
            leaves += [qw, kw]
            y = torch.cat([ref.rmsnorm(x[:, :n_q], qw, eps), ref.rmsnorm(x[:, n_q:], kw, eps)], 1)
        y = ref.apply_rope(y, pos, inv_freq)
        dy = dqkv[:, : (n_q + n_k) * hd].view(T, n_q + n_k, hd).float()
        grads = torch.autograd.grad(y, leaves, dy)
    dqkv[:, : (n_q + n_k) * hd].copy_(grads[0].reshape(T, -1).to(dqkv.dtype))
    if q_w is not None:
        if dq_w is not None:
            dq_w.add_(grads[1].to(dq_w.dtype))
        if dk_w is not None:
            dk_w.add_(grads[2].to(dk_w.dtype))


# -------------------------------------------------------------- attention
from .attention import attention_bwd, attention_fwd  # noqa: E402

# ----------------------------------------------------------------- AdamW
def adamw_flat_(p, g, m, v, p16, *, lr, betas, eps, weight_decay, step, gscale=None, gscale_host=1.0):
    """One fused AdamW step over flat fp32 buffers, writing the bf16 shadow."""
    if not p.is_cuda:
        b1, b2 = betas
        gg = g * gscale_host * (gscale if gscale is not None else 1.0)
        m.mul_(b1).add_(gg, alpha=1 - b1)
        v.mul_(b2).addcmul_(gg, gg, value=1 - b2)
        p.mul_(1 - lr * weight_decay)
        bc1 = 1 - b1**step
        bc2 = 1 - b2**step
        p.addcdiv_(m, (v.sqrt() / math.sqrt(bc2)).add_(eps), value=-lr / bc1)
        if p16 is not None:
            p16.copy_(p)
        return
    ext().adamw_step(p, g, m, v, p16, lr, betas[0], betas[1], eps, weight_decay, step, gscale, gscale_host)


Q8_BLOCK = 256


def q8m_decode(c: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    """8-bit signed log code -> value (block scale ``a`` broadcast per 256)."""
    mag = c.abs().float()
    v = a * torch.exp2((mag - 127.0) * 0.125)
    return torch.where(c == 0, torch.zeros_like(v), torch.where(c < 0, -v, v))


def q8m_encode(x: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    r = x.abs() / a.clamp_min(1e-38)
    c = torch.round(127.0 + 8.0 * torch.log2(r.clamp_min(1e-38)))
    small = torch.where(r >= 0.5 * 2.0 ** (-126 * 0.125), 1.0, 0.0)
    c = torch.where(c < 1, small, c).clamp(max=127)
    c = torch.where((a > 0) & (x != 0), c, torch.zeros_like(c))
    return torch.where(x < 0, -c, c).to(torch.int8)


def q8v_decode(c: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    v = a * torch.exp2((c.float() - 255.0) * 0.0625)
    return torch.where(c == 0, torch.zeros_like(v), v)


def q8v_encode(x: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    r = x / a.clamp_min(1e-38)
    c = torch.round(255.0 + 16.0 * torch.log2(r.clamp_min(1e-38)))
    small = torch.where(r >= 0.5 * 2.0 ** (-254 * 0.0625), 1.0, 0.0)
    c = torch.where(c < 1, small, c).clamp(max=255)
    c = torch.where((a > 0) & (x > 0), c, torch.zeros_like(c))
    return c.to(torch.uint8)


def q8_dequant_moments(m8, v8, am, av):
    """fp32 (m, v) of 8-bit block-coded moments (checkpoint re-sharding)."""
    n = m8.numel()
    nb = (n + Q8_BLOCK - 1) // Q8_BLOCK
    idx = torch.arange(n, device=m8.device) // Q8_BLOCK
    return q8m_decode(m8, am[:nb][idx]), q8v_decode(v8, av[:nb][idx])


def q8_quant_moments(m, v):
    """8-bit codes and block scales of fp32 moments (m, v)."""
    n = m.numel()
    nb = (n + Q8_BLOCK - 1) // Q8_BLOCK
    pad = nb * Q8_BLOCK - n
    mb = torch.nn.functional.pad(m.float(), (0, pad)).view(nb, Q8_BLOCK)
    vb = torch.nn.functional.pad(v.float(), (0, pad)).view(nb, Q8_BLOCK)
    am, av = mb.abs().amax(1), vb.amax(1)
    return (q8m_encode(mb, am[:, None]).reshape(-1)[:n], q8v_encode(vb, av[:, None]).reshape(-1)[:n], am, av)


def adamw8_flat_(p, g, m8, v8, am, av, p16, *, lr, betas, eps, weight_decay, step, gscale=None, gscale_host=1.0):
    """AdamW with 8-bit block-scaled log-coded moments (csrc/kernels.cu
    ``adamw8_kernel``); the CPU branch is the same math in float32 torch."""
    if p.is_cuda:
        ext().adamw8_step(p, g, m8, v8, am, av, p16, lr, betas[0], betas[1], eps, weight_decay, step, gscale,
                          gscale_host)
        return
    b1, b2 = betas
    n = p.numel()
    nb = (n + Q8_BLOCK - 1) // Q8_BLOCK
    pad = nb * Q8_BLOCK - n

    def blocks(t, fill=0):
        return torch.nn.functional.pad(t, (0, pad), value=fill).view(nb, Q8_BLOCK)

    gg = blocks(g.float() * gscale_host * (float(gscale) if gscale is not None else 1.0))
    m = b1 * q8m_decode(blocks(m8), am[:nb, None]) + (1 - b1) * gg
    v = b2 * q8v_decode(blocks(v8), av[:nb, None]) + (1 - b2) * gg * gg
    bc1, bc2 = 1 - b1**step, 1 - b2**step
    pp = blocks(p) * (1 - lr * weight_decay) - (lr / bc1) * m / (v.sqrt() / math.sqrt(bc2) + eps)
    valid = torch.ones(nb * Q8_BLOCK, dtype=torch.bool)
    if pad:
        valid[n:] = False
    valid = valid.view(nb, Q8_BLOCK)
    m = torch.where(valid, m, torch.zeros_like(m))
    v = torch.where(valid, v, torch.zeros_like(v))
    amax_m = m.abs().amax(1)
    amax_v = v.amax(1)
    p.copy_(pp.reshape(-1)[:n])
    m8.copy_(q8m_encode(m, amax_m[:, None]).reshape(-1)[:n])
    v8.copy_(q8v_encode(v, amax_v[:, None]).reshape(-1)[:n])
    am[:nb] = amax_m
    av[:nb] = amax_v
    if p16 is not None:
        p16.copy_(p)


def sumsq_(x, out):
    if not x.is_cuda:
        out[0] += x.double().pow(2).sum().float()
        out[1] += (~torch.isfinite(x)).sum().float()
        return
    ext().sumsq(x, out)
