"""DeepSeek-V4 building blocks: RMS norms, the two interleaved rotary
tables and the manifold-constrained hyper-connections (reference
trainer/models/deepseek_v4/hyperconnections.py, rotary.py).

Hyper-connections (mHC).  The residual is ``hc`` parallel streams
``X[t, i, :]``.  Around every sub-layer one linear map of the
RMS-normalised, flattened streams gives three gates:

* ``pre[i]  = sigmoid(a_pre * z_pre[i] + b_pre[i]) + eps``  collapses the
  streams into the sub-layer input ``sum_i pre[i] X_i``;
* ``post[i] = 2 sigmoid(a_post * z_post[i] + b_post[i])`` spreads the
  sub-layer output back over the streams;
* ``comb = Sinkhorn(a_comb * Z_comb + B_comb)`` (``hc x hc``), a doubly
  stochastic remix: softmax over the last axis, then alternating column /
  row normalisation, ``hc_sinkhorn_iters`` rounds in all.

``X'_j = post[j] * y + sum_i comb[i, j] X_i``.  Gates and Sinkhorn run in
fp32.  RoPE: each head is ``[nope | rope]``; the rope part rotates adjacent
channel pairs ``(x_{2k}, x_{2k+1})`` by ``pos * inv_freq[k]``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .config import DeepseekV4Config


class RMSNorm(nn.Module):
    """Weighted RMS norm computed in fp32."""

    def __init__(self, width: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


def rms_unweighted(x: Tensor, eps: float, out_dtype: torch.dtype | None = None) -> Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(out_dtype or x.dtype)


# ----------------------------------------------------------------- rotary
def _inv_freq(params: dict, head_dim: int) -> tuple[Tensor, float]:
    """Inverse frequencies of the rotary slice and the cos/sin scale."""
    dim = int(head_dim * params.get("partial_rotary_factor", 1.0))
    base = float(params["rope_theta"])
    inv = 1.0 / base ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    kind = params.get("rope_type", "default")
    if kind == "default":
        return inv.float(), 1.0
    if kind == "linear":
        return (inv / float(params["factor"])).float(), 1.0
    if kind == "yarn":
        # YaRN (Peng et al. 2023, "YaRN: Efficient Context Window Extension"):
        # dimensions whose wavelength is short keep their frequency, long ones
        # are interpolated by `factor`, with a linear ramp between the
        # dimensions that complete beta_fast and beta_slow turns over the
        # original context.
        factor = float(params["factor"])
        orig = float(params.get("original_max_position_embeddings", 4096))
        beta_fast, beta_slow = float(params.get("beta_fast", 32.0)), float(params.get("beta_slow", 1.0))

        def dim_for(turns: float) -> float:
            return dim * math.log(orig / (turns * 2 * math.pi)) / (2 * math.log(base))

        lo = max(math.floor(dim_for(beta_fast)), 0)
        hi = min(math.ceil(dim_for(beta_slow)), dim - 1)
        if hi == lo:
            hi += 0.001
        ramp = ((torch.arange(dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
        extrapolate = 1.0 - ramp  # 1: keep the original frequency
        inv = (inv / factor) * (1 - extrapolate) + inv * extrapolate
        scale = params.get("attention_factor")
        if scale is None:
            scale = 0.1 * math.log(factor) + 1.0
        return inv.float(), float(scale)
    raise ValueError(f"rope type {kind!r} is not supported (default, linear, yarn)")


class DualRotary(nn.Module):
    """cos / sin at half width (one per channel pair) for the ``main`` and
    ``compress`` tables."""

    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        self.config = config
        self.kinds = [k for k, v in config.rope_parameters.items() if isinstance(v, dict)]
        self.scale: dict[str, float] = {}
        for k in self.kinds:
            inv, sc = _inv_freq(config.rope_parameters[k], config.head_dim)
            self.register_buffer(f"{k}_inv_freq", inv, persistent=False)
            self.scale[k] = sc

    def reset_tables(self) -> None:
        for k in self.kinds:
            inv, sc = _inv_freq(self.config.rope_parameters[k], self.config.head_dim)
            getattr(self, f"{k}_inv_freq").copy_(inv)
            self.scale[k] = sc

    @torch.no_grad()
    def forward(self, positions: Tensor, kind: str, dtype: torch.dtype) -> tuple[Tensor, Tensor]:
        """positions [..., n] -> cos, sin [..., n, rope_dim / 2]."""
        inv = getattr(self, f"{kind}_inv_freq").to(positions.device)
        ang = positions.float().unsqueeze(-1) * inv
        return (ang.cos() * self.scale[kind]).to(dtype), (ang.sin() * self.scale[kind]).to(dtype)


def rope_interleaved(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate the trailing ``2 * cos.shape[-1]`` channels of ``x`` as adjacent
    pairs; cos / sin broadcast against ``x[..., :, pairs]`` (callers insert
    the head axis)."""
    r = 2 * cos.shape[-1]
    keep, rot = x[..., :-r], x[..., -r:]
    a, b = rot.float()[..., 0::2], rot.float()[..., 1::2]
    c, s = cos.float(), sin.float()
    out = torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2).to(x.dtype)
    return torch.cat((keep, out), dim=-1)


# ------------------------------------------------------- hyper-connections
def sinkhorn(logits: Tensor, iters: int, eps: float) -> Tensor:
    m = torch.softmax(logits, dim=-1) + eps
    m = m / (m.sum(-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        m = m / (m.sum(-1, keepdim=True) + eps)
        m = m / (m.sum(-2, keepdim=True) + eps)
    return m


class HyperConnection(nn.Module):
    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        self.hc = config.hc_mult
        self.iters = config.hc_sinkhorn_iters
        self.eps = config.hc_eps
        self.norm_eps = config.rms_norm_eps
        self.fn = nn.Parameter(torch.empty((2 + self.hc) * self.hc, self.hc * config.hidden_size))
        self.base = nn.Parameter(torch.empty((2 + self.hc) * self.hc))
        self.scale = nn.Parameter(torch.empty(3))  # pre, post, comb

    def reset_parameters(self, std: float) -> None:
        nn.init.normal_(self.fn, std=std)
        nn.init.zeros_(self.base)
        nn.init.ones_(self.scale)

    def forward(self, streams: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """streams [..., hc, H] -> (post [..., hc], comb [..., hc, hc], collapsed [..., H])."""
        hc = self.hc
        z = F.linear(rms_unweighted(streams.flatten(-2), self.norm_eps, torch.float32), self.fn.float())
        zp, zq, zc = z.split([hc, hc, hc * hc], dim=-1)
        bp, bq, bc = self.base.float().split([hc, hc, hc * hc])
        sp, sq, sc = self.scale.float().unbind(0)
        pre = torch.sigmoid(zp * sp + bp) + self.eps
        post = 2.0 * torch.sigmoid(zq * sq + bq)
        comb = sinkhorn(zc.unflatten(-1, (hc, hc)) * sc + bc.view(hc, hc), self.iters, self.eps)
        collapsed = (pre.unsqueeze(-1) * streams).sum(-2).to(streams.dtype)
        return post, comb, collapsed

    @staticmethod
    def merge(post: Tensor, comb: Tensor, out: Tensor, streams: Tensor) -> Tensor:
        dt = streams.dtype
        return post.to(dt).unsqueeze(-1) * out.unsqueeze(-2) + comb.to(dt).transpose(-1, -2) @ streams


class HyperHead(nn.Module):
    """Final collapse of the streams (before the last norm)."""

    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        self.hc = config.hc_mult
        self.eps = config.hc_eps
        self.norm_eps = config.rms_norm_eps
        self.hc_fn = nn.Parameter(torch.empty(self.hc, self.hc * config.hidden_size))
        self.hc_base = nn.Parameter(torch.empty(self.hc))
        self.hc_scale = nn.Parameter(torch.empty(1))

    def reset_parameters(self, std: float) -> None:
        nn.init.normal_(self.hc_fn, std=std)
        nn.init.zeros_(self.hc_base)
        nn.init.ones_(self.hc_scale)

    def forward(self, streams: Tensor) -> Tensor:
        z = F.linear(rms_unweighted(streams.flatten(-2), self.norm_eps, torch.float32), self.hc_fn.float())
        pre = torch.sigmoid(z * self.hc_scale.float() + self.hc_base.float()) + self.eps
        return (pre.unsqueeze(-1) * streams).sum(-2).to(streams.dtype)
