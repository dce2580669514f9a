"""Qwen3-MoE sparse MLP block: router, top-k routing, expert SwiGLU FFNs.

GPU path (``MoEBlock``), inside the recompute-based decoder layer:

    h2 = rmsnorm(x2)                         logits = h2 Wr^T            (fp32)
    p  = softmax(logits); (w, e) = topk(p)   w /= sum(w) if norm_topk_prob
    token copies are laid out expert-by-expert in a buffer whose expert
    segments are padded to 128 rows, so every 128-row GEMM tile belongs to one
    expert; the expert FFNs run as grouped tcgen05 GEMMs (M-grouped: the tile's
    expert selects its weight block) and the weight gradients as K-grouped
    GEMMs over each expert's token segment, accumulated in fp32 straight into
    the flat gradient buffer.
    out = x2 + sum_k w_k * expert_{e_k}(h2)

Auxiliary load-balance loss (Switch form, ``router_aux_loss_coef``):
    L_aux = E * sum_e f_e * P_e,  f_e = share of the T*k assignments routed to
    e, P_e = mean router probability of e; its gradient (f_e treated as a
    constant) is injected into the router gradient in the block's backward,
    scaled by ``aux_loss_scale`` (set by the trainer per micro-batch).

``moe_reference`` is the float32 eager formulation (the CPU path and the
oracle), matching HF ``Qwen3MoeSparseMoeBlock`` used by the reference
(trainer/moe.py:241-272, routing metrics :387-436).

Expert parallelism (EP) exchanges token copies with NCCL all-to-all
(``ep_group``); the counts are exchanged first so every rank knows its
receive layout (trainer/moe.py:174-233).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref

PAD = 128


def moe_reference(h: torch.Tensor, router_w: torch.Tensor, gu_w: torch.Tensor, down_w: torch.Tensor, cfg):
    """Returns (out [T, H], aux_loss scalar, stats)."""
    T = h.shape[0]
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    logits = h.float() @ router_w.float().t()
    probs = torch.softmax(logits, -1)
    topv, topi = torch.topk(probs, k, dim=-1)
    if cfg.norm_topk_prob:
        topv = topv / topv.sum(-1, keepdim=True)
    out = torch.zeros(T, h.shape[1], dtype=torch.float32, device=h.device)
    for e in range(E):
        sel = (topi == e)
        tok = sel.any(-1).nonzero().flatten()
        if tok.numel() == 0:
            continue
        w = (topv * sel).sum(-1)[tok]
        y = ref.swiglu(h[tok].float() @ gu_w[e].float().t()) @ down_w[e].float().t()
        out.index_add_(0, tok, y * w[:, None])
    counts = torch.bincount(topi.flatten(), minlength=E).float()
    f = counts / (T * k)
    P = probs.mean(0)
    aux = E * (f * P).sum()
    return out.to(h.dtype), aux, {"counts": counts}


class Routing:
    """Padded expert layout of the T*k token copies of a micro-batch."""

    def __init__(self, topi: torch.Tensor, E: int, pad: int = PAD):
        T, k = topi.shape
        dev = topi.device
        flat = topi.reshape(-1)
        counts = torch.bincount(flat, minlength=E)
        cl = counts.tolist()  # host sync: the padded layout sizes the grouped GEMM grid
        padded = [(c + pad - 1) // pad * pad for c in cl]
        starts = [0] * E
        acc = 0
        for e in range(E):
            starts[e] = acc
            acc += padded[e]
        self.R = max(acc, pad)
        self.counts = counts
        order = torch.argsort(flat, stable=True)
        rank_in = torch.empty_like(order)
        cum = torch.zeros(E + 1, dtype=torch.long, device=dev)
        cum[1:] = counts.cumsum(0)
        sorted_e = flat[order]
        rank_in[order] = torch.arange(flat.numel(), device=dev) - cum[sorted_e]
        start_t = torch.tensor(starts, dtype=torch.long, device=dev)
        self.pos = start_t[flat] + rank_in  # row of each (token, slot) copy in the padded buffer
        self.tok = torch.arange(T, device=dev).repeat_interleave(k)
        tiles = []
        for e in range(E):
            tiles += [e] * (padded[e] // pad)
        if not tiles:
            tiles = [0]
        self.tile_group = torch.tensor(tiles, dtype=torch.int32, device=dev)
        self.k_start = torch.tensor(starts, dtype=torch.int32, device=dev)
        self.k_len = torch.tensor(padded, dtype=torch.int32, device=dev)
        self.E = E


class DeviceRouting:
    """The ``Routing`` layout built on the device (``moe_layout`` /
    ``moe_copy_rows`` kernels): no host round trip, so a layer needs no
    synchronisation and can be captured in a CUDA graph.  The row buffers are
    sized for the worst case (every copy plus a full padding tile per expert);
    tiles past the used rows carry group -1 and the grouped GEMMs skip them."""

    def __init__(self, topi: torch.Tensor, counts: torch.Tensor, E: int, pad: int = PAD):
        T, k = topi.shape
        dev = topi.device
        m = ops.ext()
        self.E = E
        self.R = max(pad, (T * k + E * (pad - 1) + pad - 1) // pad * pad)
        self.counts = counts
        self.base = torch.empty(E, dtype=torch.int64, device=dev)
        self.tile_group = torch.empty(self.R // pad, dtype=torch.int32, device=dev)
        self.k_start = torch.empty(E, dtype=torch.int32, device=dev)
        self.k_len = torch.empty(E, dtype=torch.int32, device=dev)
        self.n_recv = torch.empty(E, dtype=torch.int32, device=dev)
        self.rows = torch.empty(1, dtype=torch.int32, device=dev)
        self.overflow = torch.empty(1, dtype=torch.int32, device=dev)
        m.moe_layout(counts, 1, 0, pad, self.R, self.base, self.tile_group, self.k_start, self.k_len, self.n_recv,
                     self.rows, self.overflow)
        self.pos = torch.empty(T * k, dtype=torch.int64, device=dev)
        self.dst_rank = torch.empty(T * k, dtype=torch.int32, device=dev)
        m.moe_copy_rows(topi.reshape(-1).contiguous(), E, E, self.base, self.pos, self.dst_rank)
        self.tok = torch.arange(T, device=dev).repeat_interleave(k)

    def scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        """[R, H] buffer with row pos[i] = x[tok[i]] and zero padding rows."""
        xs = torch.empty(self.R, x.shape[1], device=x.device, dtype=x.dtype)
        xs.index_copy_(0, self.pos, x.index_select(0, self.tok))
        ops.ext().moe_zero_pad(xs, self.k_start, self.k_len, self.n_recv, self.overflow)
        return xs

    def scatter_copies(self, rows: torch.Tensor) -> torch.Tensor:
        """[R, H] buffer with row pos[i] = rows[i] ((token, slot) order) and zero padding."""
        out = torch.empty(self.R, rows.shape[1], device=rows.device, dtype=rows.dtype)
        out.index_copy_(0, self.pos, rows)
        ops.ext().moe_zero_pad(out, self.k_start, self.k_len, self.n_recv, self.overflow)
        return out


def moe_metrics(model) -> dict[str, float]:
    """moe/max_vio (mean over layers of (max expert load - mean) / mean),
    its max over layers, and moe/routing_confidence (mean selected top-k
    probability mass) of the last forward (reference trainer/moe.py:387-436);
    one host transfer for all layers."""
    stats = [layer.moe.last_stats for layer in getattr(model, "layers", [])
             if getattr(layer, "moe", None) is not None and layer.moe.last_stats is not None]
    if not stats:
        return {}
    st = torch.stack(stats).float().cpu()
    return {"moe/max_vio": float(st[:, 0].mean()), "moe/max_vio/max": float(st[:, 0].max()),
            "moe/routing_confidence": float(st[:, 1].mean())}


class MoEBlock:
    """Sparse MLP of one decoder layer (GPU path and the CPU fallbacks of the
    same ops).  With ``ep_size > 1`` this rank holds experts
    [ep_rank * E/ep, (ep_rank + 1) * E/ep) and token copies travel to their
    expert's rank and back (dispatch / combine); gradients take the same
    route in reverse.  ``ep_group`` is set by the model before each forward."""

    def __init__(self, cfg, layer_idx: int, ep_size: int = 1, ep_rank: int = 0):
        self.cfg = cfg
        self.layer = layer_idx
        self.ep_group = None
        self.ep_fabric = None  # parallel.ep_fabric.FabricEP: dispatch / combine over peer memory
        self.ep_size = ep_size
        self.ep_rank = ep_rank
        self.E_loc = cfg.num_experts // ep_size
        self.aux_loss_scale = 0.0
        self.last_counts = None
        self.last_stats = None  # device [max_vio, routing confidence] of the last forward
        self.router_logits_bf16 = False  # model.moe_router_dtype == 'none' (set by apply_model_options)

    # ------------------------------------------------------------ shared
    def _route(self, h2, P):
        """Router logits GEMM, then softmax / top-k / weights / per-expert
        counts in one device kernel (``moe_route``).  With
        model.moe_router_dtype 'none' the logits are rounded to bf16 first (a
        gate in the model dtype); 'float32' keeps the fp32 GEMM output."""
        cfg = self.cfg
        logits = ops.gemm(h2, P["router_w"], epi=ops.EPI_F32)
        k, E = cfg.num_experts_per_tok, cfg.num_experts
        T = logits.shape[0]
        if logits.is_cuda:
            dev = logits.device
            probs = torch.empty(T, E, device=dev, dtype=torch.float32)
            topi = torch.empty(T, k, device=dev, dtype=torch.int64)
            topv = torch.empty(T, k, device=dev, dtype=torch.float32)
            w = torch.empty(T, k, device=dev, dtype=torch.float32)
            s = torch.empty(T, 1, device=dev, dtype=torch.float32)
            counts = torch.zeros(E, device=dev, dtype=torch.int32)
            ops.ext().moe_route(logits.contiguous(), k, bool(cfg.norm_topk_prob), bool(self.router_logits_bf16),
                                probs, topi, topv, w, s, counts)
        else:
            if self.router_logits_bf16:
                logits = logits.to(torch.bfloat16).float()
            probs = torch.softmax(logits, -1)
            topv, topi = torch.topk(probs, k, dim=-1)
            s = topv.sum(-1, keepdim=True)
            w = topv / s if cfg.norm_topk_prob else topv
            counts = torch.bincount(topi.reshape(-1), minlength=E).to(torch.int32)
        self._counts = counts
        return probs, topv, topi, s, w

    def _note_stats(self, counts: torch.Tensor, s: torch.Tensor) -> None:
        c = counts.float()
        mean = c.mean().clamp_min(1e-9)
        self.last_counts = counts
        self.last_stats = torch.stack([(c.max() - mean) / mean, s.float().mean()])

    def _local_routing(self, topi):
        if topi.is_cuda:
            return DeviceRouting(topi, self._counts, self.cfg.num_experts)
        return Routing(topi, self.cfg.num_experts)

    def _experts(self, x, P, rt):
        """Expert FFNs of this rank over the rows ``x[rt.tok]`` laid out by ``rt``."""
        cfg = self.cfg
        E, H, Ie = self.E_loc, cfg.hidden_size, cfg.moe_intermediate_size
        if isinstance(rt, DeviceRouting):
            xs = rt.scatter_rows(x)
        else:
            xs = torch.zeros(rt.R, H, device=x.device, dtype=x.dtype)
            xs.index_copy_(0, rt.pos, x.index_select(0, rt.tok))
        gu = torch.empty(rt.R, 2 * Ie, device=x.device, dtype=x.dtype)
        ops.gemm_grouped(xs, False, P["exp_gu_w"].view(E * 2 * Ie, H), False, gu, 1, rt.R, 2 * Ie, H, rt.tile_group,
                         2 * Ie, E * 2 * Ie, None, None, E, ops.EPI_BF16, 1.0)
        a = ops.swiglu_fwd(gu)
        y = torch.empty(rt.R, H, device=x.device, dtype=x.dtype)
        ops.gemm_grouped(a, False, P["exp_down_w"].view(E * H, Ie), False, y, 1, rt.R, H, Ie, rt.tile_group, H, E * H,
                         None, None, E, ops.EPI_BF16, 1.0)
        return xs, gu, a, y

    def _experts_bwd(self, dy, c, P, G, out=None):
        """Backward of ``_experts`` from the padded-row gradient ``dy`` [R, H];
        accumulates the expert weight gradients, returns d(xs) [R, H]."""
        cfg = self.cfg
        E, H, Ie = self.E_loc, cfg.hidden_size, cfg.moe_intermediate_size
        rt: Routing = c["rt"]
        da = torch.empty(rt.R, Ie, device=dy.device, dtype=dy.dtype)
        ops.gemm_grouped(dy, False, P["exp_down_w"].view(E * H, Ie), True, da, 1, rt.R, Ie, H, rt.tile_group, H, E * H,
                         None, None, E, ops.EPI_BF16, 1.0)
        if G.get("exp_down_w") is not None:
            ops.gemm_grouped(dy, True, c["a"], True, G["exp_down_w"].view(E * H, Ie), 2, H, Ie, rt.R, None, 0, 0,
                             rt.k_start, rt.k_len, E, ops.EPI_F32_ACC, 1.0)
        dgu = ops.swiglu_bwd(c["gu"], da)
        del da
        if G.get("exp_gu_w") is not None:
            ops.gemm_grouped(dgu, True, c["xs"], True, G["exp_gu_w"].view(E * 2 * Ie, H), 2, 2 * Ie, H, rt.R, None, 0,
                             0, rt.k_start, rt.k_len, E, ops.EPI_F32_ACC, 1.0)
        dxs = out if out is not None else torch.empty(rt.R, H, device=dy.device, dtype=dy.dtype)
        ops.gemm_grouped(dgu, False, P["exp_gu_w"].view(E * 2 * Ie, H), True, dxs, 1, rt.R, H, 2 * Ie, rt.tile_group,
                         2 * Ie, E * 2 * Ie, None, None, E, ops.EPI_BF16, 1.0)
        return dxs

    # ------------------------------------------------------- dispatch / combine
    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.ep_group)
        return out

    def _dispatch(self, h2, topi):
        """Send every (token, slot) copy to its expert's rank.  Returns the
        plan (orders and split sizes) and the received rows, which arrive
        grouped by source rank, then by local expert."""
        T, k = topi.shape
        ep, El = self.ep_size, self.E_loc
        e = topi.reshape(-1)
        order = torch.argsort(e, stable=True)  # by destination rank, then local expert
        cnt = torch.bincount(e, minlength=self.cfg.num_experts)
        recv = torch.empty_like(cnt)
        self._a2a(recv, cnt, None, None)  # recv[src * El + el]: copies from src for my expert el
        send_h = cnt.view(ep, El).sum(1).tolist()
        recv_mat = recv.view(ep, El)
        recv_h = recv_mat.sum(1).tolist()  # host sync: the split sizes size the transfers
        tok = torch.arange(T, device=h2.device).repeat_interleave(k)[order]
        x_recv = h2.new_empty(sum(recv_h), h2.shape[1])
        self._a2a(x_recv, h2.index_select(0, tok), recv_h, send_h)
        el = torch.repeat_interleave(torch.arange(El, device=h2.device).repeat(ep), recv_mat.reshape(-1))
        return dict(order=order, tok=tok, send=send_h, recv=recv_h, counts=cnt), x_recv, el

    def _combine(self, y_recv, plan, T, k):
        """Return expert outputs to their tokens' ranks, in (token, slot) order."""
        y_send = y_recv.new_empty(T * k, y_recv.shape[1])
        self._a2a(y_send, y_recv, plan["send"], plan["recv"])
        y_copy = torch.empty_like(y_send)
        y_copy[plan["order"]] = y_send
        return y_copy

    # ------------------------------------------------------------ forward
    def forward(self, x2, P, save: bool):
        cfg = self.cfg
        T = x2.shape[0]
        k = cfg.num_experts_per_tok
        h2, rstd2, _ = ops.rmsnorm_fwd(x2, P["post_norm"], cfg.rms_eps)
        probs, topv, topi, s, w = self._route(h2, P)
        if self.ep_fabric is not None and self.ep_size > 1:
            return self._forward_fabric(x2, P, save, h2, rstd2, probs, topv, topi, s, w)
        if self.ep_size > 1:
            plan, x_recv, el = self._dispatch(h2, topi)
            rt = Routing(el.view(-1, 1), self.E_loc)
            xs, gu, a, y = self._experts(x_recv, P, rt)
            y_copy = self._combine(y.index_select(0, rt.pos), plan, T, k)
            counts = plan["counts"]
        else:
            plan = None
            rt = self._local_routing(topi)
            xs, gu, a, y = self._experts(h2, P, rt)
            y_copy = y.index_select(0, rt.pos)
            counts = rt.counts
        contrib = y_copy.float() * w.reshape(-1, 1)
        out = (x2.float() + contrib.view(T, k, -1).sum(1)).to(x2.dtype)
        f = counts.float() / (T * k)
        self._note_stats(counts, s)
        cache = None
        if save:
            cache = dict(h2=h2, rstd2=rstd2, probs=probs, topv=topv, topi=topi, s=s, w=w, rt=rt, xs=xs, gu=gu, a=a,
                         y_copy=y_copy, f=f, plan=plan)
        return out, cache

    # ------------------------------------------- expert parallel over peer memory
    def _fabric_experts(self, xs, P, fp, y_out):
        cfg = self.cfg
        E, H, Ie = self.E_loc, cfg.hidden_size, cfg.moe_intermediate_size
        gu = torch.empty(fp.R, 2 * Ie, device=xs.device, dtype=xs.dtype)
        ops.gemm_grouped(xs, False, P["exp_gu_w"].view(E * 2 * Ie, H), False, gu, 1, fp.R, 2 * Ie, H, fp.tile_group,
                         2 * Ie, E * 2 * Ie, None, None, E, ops.EPI_BF16, 1.0)
        a = ops.swiglu_fwd(gu)
        ops.gemm_grouped(a, False, P["exp_down_w"].view(E * H, Ie), False, y_out, 1, fp.R, H, Ie, fp.tile_group, H,
                         E * H, None, None, E, ops.EPI_BF16, 1.0)
        return gu, a

    def _forward_fabric(self, x2, P, save, h2, rstd2, probs, topv, topi, s, w):
        cfg = self.cfg
        T, k = x2.shape[0], cfg.num_experts_per_tok
        fe = self.ep_fabric
        fp = fe.plan(topi, self._counts)
        xs = fe.dispatch("xs", h2, fp)  # rows land directly in the owner's padded expert layout
        gu, a = self._fabric_experts(xs, P, fp, fe.view("y", fp.R))
        out = torch.empty_like(x2)
        fe.combine("y", fp, k, w, x2, out)  # out = x2 + sum_k w_k y_k, read from the owners
        f = fp.counts.float() / (T * k)
        self._note_stats(fp.counts, s)
        cache = None
        if save:
            y_copy = fe.gather_copies("y", fp, T, k)
            cache = dict(h2=h2, rstd2=rstd2, probs=probs, topv=topv, topi=topi, s=s, w=w, rt=fp, xs=xs.clone(),
                         gu=gu, a=a, y_copy=y_copy, f=f, plan=None, fplan=fp)
        return out, cache

    # ------------------------------------------------------------ backward
    def backward(self, dout, x2, c, P, G):
        cfg = self.cfg
        H, k = cfg.hidden_size, cfg.num_experts_per_tok
        T = x2.shape[0]
        rt: Routing = c["rt"]
        if c.get("fplan") is not None:
            fe, fp = self.ep_fabric, c["fplan"]
            dy = fe.dispatch("dy", dout.contiguous(), fp, scale=c["w"].reshape(-1).float().contiguous())
            self._experts_bwd(dy, c, P, G, out=fe.view("dxs", fp.R))
            dh2 = torch.empty(T, H, device=dout.device, dtype=torch.float32)
            fe.combine("dxs", fp, k, None, None, dh2)
            tok_copy = torch.arange(T, device=dout.device).repeat_interleave(k)
            dw = (dout.index_select(0, tok_copy).float() * c["y_copy"].float()).sum(-1).view(T, k)
            return self._router_bwd(dout, x2, c, P, G, dw, dh2)
        tok_copy = torch.arange(T, device=dout.device).repeat_interleave(k)
        dout_rows = dout.index_select(0, tok_copy).float()  # [T*k, H] in (token, slot) order
        w = c["w"].reshape(-1, 1)
        dw = (dout_rows * c["y_copy"].float()).sum(-1).view(T, k)
        dy_copy = (dout_rows * w).to(dout.dtype)
        plan = c["plan"]
        if plan is not None:
            dy_recv = dout.new_empty(sum(plan["recv"]), H)
            self._a2a(dy_recv, dy_copy[plan["order"]], plan["recv"], plan["send"])
            dy = torch.zeros(rt.R, H, device=dout.device, dtype=dout.dtype)
            dy.index_copy_(0, rt.pos, dy_recv)
        elif isinstance(rt, DeviceRouting):
            dy = rt.scatter_copies(dy_copy)
        else:
            dy = torch.zeros(rt.R, H, device=dout.device, dtype=dout.dtype)
            dy.index_copy_(0, rt.pos, dy_copy)
        dxs = self._experts_bwd(dy, c, P, G)
        dh2 = torch.zeros(T, H, device=dout.device, dtype=torch.float32)
        if plan is not None:
            dx_send = dout.new_empty(T * k, H)
            self._a2a(dx_send, dxs.index_select(0, rt.pos), plan["send"], plan["recv"])
            dh2.index_add_(0, plan["tok"], dx_send.float())
        else:
            dh2.index_add_(0, rt.tok, dxs.index_select(0, rt.pos).float())
        del dxs
        return self._router_bwd(dout, x2, c, P, G, dw, dh2)

    def _router_bwd(self, dout, x2, c, P, G, dw, dh2):
        cfg = self.cfg
        T = x2.shape[0]
        # router: top-k weights (optionally renormalised) and the aux loss
        if cfg.norm_topk_prob:
            wv = c["w"]
            dv = (dw - (dw * wv).sum(-1, keepdim=True)) / c["s"]
        else:
            dv = dw
        probs = c["probs"]
        dprobs = torch.zeros_like(probs).scatter_(1, c["topi"], dv)
        if self.aux_loss_scale:
            dprobs += self.aux_loss_scale * cfg.num_experts * c["f"][None, :] / T
        dlogits = probs * (dprobs - (dprobs * probs).sum(-1, keepdim=True))
        dl16 = dlogits.to(dout.dtype).contiguous()
        if G.get("router_w") is not None:
            ops.gemm(dl16, c["h2"], a_mn=True, b_mn=True, out=G["router_w"], epi=ops.EPI_F32_ACC)
        dh2 += ops.gemm(dl16, P["router_w"], b_mn=True).float()
        return ops.rmsnorm_bwd(x2, P["post_norm"], c["rstd2"], dh2.to(dout.dtype), dres=dout, dw=G.get("post_norm"))

    # ------------------------------------------------------------ generator
    @torch.no_grad()
    def infer(self, h2, x, P):
        cfg = self.cfg
        T = h2.shape[0]
        k = cfg.num_experts_per_tok
        if not h2.is_cuda and self.ep_size == 1:
            out, _, _ = moe_reference(h2, P["router_w"], P["exp_gu_w"], P["exp_down_w"], cfg)
            return x + out
        probs, topv, topi, s, w = self._route(h2, P)
        if self.ep_fabric is not None and self.ep_size > 1:
            fe = self.ep_fabric
            fp = fe.plan(topi, self._counts)
            xs = fe.dispatch("xs", h2, fp)
            self._fabric_experts(xs, P, fp, fe.view("y", fp.R))
            out = torch.empty_like(x)
            return fe.combine("y", fp, k, w, x, out)
        if self.ep_size > 1:
            plan, x_recv, el = self._dispatch(h2, topi)
            rt = Routing(el.view(-1, 1), self.E_loc)
            _, _, _, y = self._experts(x_recv, P, rt)
            y_copy = self._combine(y.index_select(0, rt.pos), plan, T, k)
        else:
            rt = self._local_routing(topi)
            _, _, _, y = self._experts(h2, P, rt)
            y_copy = y.index_select(0, rt.pos)
        contrib = y_copy.float() * w.reshape(-1, 1)
        return (x.float() + contrib.view(T, k, -1).sum(1)).to(x.dtype)
