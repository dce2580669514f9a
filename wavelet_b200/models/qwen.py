"""Qwen2 / Qwen3 / Qwen3-MoE causal LM on flat parameters.

GPU path: embedding -> N x ``DecoderLayerFn`` (fused kernels, recompute) ->
final RMSNorm -> chunked LM head (``ops.lm_head``).  CPU path: the same math
with plain PyTorch float32 ops and autograd (used by the CPU/gloo plumbing
configuration and as the numerics oracle).

Parity: the reference trains Hugging Face ``Qwen2ForCausalLM`` /
``Qwen3ForCausalLM`` / ``Qwen3MoeForCausalLM`` loaded in trainer/model.py:536;
parameter names map 1:1 to the HF names (``models.hf_io``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref
from .config import ArchConfig
from .layers import BatchCtx, DecoderLayerFn, EmbeddingFn, FinalNormFn
from .params import FlatParams, ParamSpec, ShardedFlatParams


def param_specs(cfg: ArchConfig) -> list[ParamSpec]:
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    std = cfg.init_std
    s: list[ParamSpec] = [ParamSpec("embed", (cfg.vocab_size, H), std=std)]
    for i in range(cfg.num_layers):
        p = f"l{i}."
        s.append(ParamSpec(p + "in_norm", (H,), "ones", False))
        s.append(ParamSpec(p + "qkv_w", (cfg.qkv_dim, H), std=std))
        if cfg.qkv_bias:
            s.append(ParamSpec(p + "qkv_b", (cfg.qkv_dim,), "zeros", False))
        if cfg.qk_norm:
            s.append(ParamSpec(p + "q_norm", (hd,), "ones", False))
            s.append(ParamSpec(p + "k_norm", (hd,), "ones", False))
        s.append(ParamSpec(p + "o_w", (H, cfg.q_dim), std=std))
        s.append(ParamSpec(p + "post_norm", (H,), "ones", False))
        if cfg.layer_is_moe(i):
            E, Ie = cfg.num_experts, cfg.moe_intermediate_size
            s.append(ParamSpec(p + "router_w", (E, H), std=std))
            s.append(ParamSpec(p + "exp_gu_w", (E, 2 * Ie, H), std=std))
            s.append(ParamSpec(p + "exp_down_w", (E, H, Ie), std=std))
        else:
            s.append(ParamSpec(p + "gu_w", (2 * I, H), std=std))
            s.append(ParamSpec(p + "down_w", (H, I), std=std))
    s.append(ParamSpec("norm", (H,), "ones", False))
    if not cfg.tie_embeddings:
        s.append(ParamSpec("lm_head", (cfg.vocab_size, H), std=std))
    return s


QUANTIZABLE = ("qkv_w", "o_w", "gu_w", "down_w")  # dense 2-D projections (NF4 for QLoRA)


def tp_local_cfg(cfg: ArchConfig, tp: int) -> ArchConfig:
    """The per-rank layer shape under tensor parallelism: heads and the MLP
    width are split, the hidden size is not."""
    if tp == 1:
        return cfg
    if cfg.num_heads % tp or cfg.num_kv_heads % tp or cfg.intermediate_size % tp:
        raise ValueError(f"tp={tp} must divide the heads ({cfg.num_heads}/{cfg.num_kv_heads}) and the MLP width")
    if cfg.is_moe:
        raise NotImplementedError("tensor parallelism with MoE layers is not supported (use expert parallelism)")
    from dataclasses import replace

    return replace(cfg, num_heads=cfg.num_heads // tp, num_kv_heads=cfg.num_kv_heads // tp,
                   intermediate_size=cfg.intermediate_size // tp)


def tp_slicers(cfg: ArchConfig, tp: int, r: int) -> dict[str, tuple]:
    """name suffix -> (full shape, fn(full) -> this rank's part).  Column-parallel
    qkv (by heads) and gate/up (by rows), row-parallel o and down (by columns):
    the Megatron split of a decoder layer."""
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    q, kv = cfg.q_dim, cfg.kv_dim
    ql, kvl, il = q // tp, kv // tp, I // tp

    def qkv_rows(full):
        return torch.cat([full[r * ql:(r + 1) * ql], full[q + r * kvl:q + (r + 1) * kvl],
                          full[q + kv + r * kvl:q + kv + (r + 1) * kvl]], 0)

    def gu_rows(full):
        return torch.cat([full[r * il:(r + 1) * il], full[I + r * il:I + (r + 1) * il]], 0)

    return {"qkv_w": ((cfg.qkv_dim, H), qkv_rows), "qkv_b": ((cfg.qkv_dim,), qkv_rows),
            "o_w": ((H, q), lambda f: f[:, r * ql:(r + 1) * ql]), "gu_w": ((2 * I, H), gu_rows),
            "down_w": ((H, I), lambda f: f[:, r * il:(r + 1) * il])}


@dataclass
class TPContext:
    group: Any
    rank: int
    size: int
    fabric: Any = None  # parallel.tp_fabric.TPFabric: fused GEMM -> all-reduce over peer memory
EXPERT_PARAMS = ("exp_gu_w", "exp_down_w")  # sharded by expert under expert parallelism


def is_expert_param(name: str) -> bool:
    return name.split(".", 1)[-1] in EXPERT_PARAMS


@dataclass
class _Layer:
    cfg: ArchConfig
    P: dict
    G: dict
    batch: BatchCtx | None = None
    moe: Any = None
    lora: dict | None = None
    offload: Any = None  # ActivationOffload when activations live in host memory
    recompute: bool = True  # activation checkpointing of this layer
    tp: Any = None  # TPContext under tensor parallelism
    index: int = 0  # position in the stack (NVTX range names)


class CausalLM:
    """A decoder-only LM whose parameters live in a ``FlatParams`` store."""

    def __init__(self, cfg: ArchConfig, flat: FlatParams, quant: dict | None = None,
                 expert_flat: FlatParams | None = None, ep: tuple[int, int] = (1, 0), tp: tuple[int, int] = (1, 0)):
        self.cfg = cfg
        self.tp_size, self.tp_rank = tp
        self.tp_group = None  # set by the trainer (NCCL / gloo group of the TP peers)
        self.tp_fabric = None  # TPFabric of the TP group (attach_tp_fabric)
        self.layer_cfg = tp_local_cfg(cfg, self.tp_size)
        self.flat = flat
        # expert parallelism: this rank's experts [ep_rank*E/ep, (ep_rank+1)*E/ep) live in expert_flat
        self.expert_flat = expert_flat
        self.ep_size, self.ep_rank = ep
        self.ep_dp_rank = 0
        self.quant = quant or {}  # name -> NF4Weight (frozen QLoRA base projections)
        self.fused_cpu = False  # run the kernel-path layer functions with their CPU fallbacks
        self.lora = None
        self.device = flat.device
        self.inv_freq = ref.rope_inv_freq(cfg.head_dim, cfg.rope_theta, device=self.device)
        self.layers: list[_Layer] = []
        for i in range(cfg.num_layers):
            pre = f"l{i}."
            names = [n for n in flat.names() if n.startswith(pre)]
            # a ZeRO-3 store binds P / G when the layer's unit is gathered
            P = {n[len(pre):]: flat.view(n) for n in names} if not flat.sharded_compute else {}
            P.update({n[len(pre):]: q for n, q in self.quant.items() if n.startswith(pre)})
            G = {n[len(pre):]: flat.grad_view(n) for n in names} if (flat.grad is not None and
                                                                     not flat.sharded_compute) else {}
            if expert_flat is not None:
                en = [n for n in expert_flat.names() if n.startswith(pre)]
                P.update({n[len(pre):]: expert_flat.view(n) for n in en})
                if expert_flat.grad is not None:
                    G.update({n[len(pre):]: expert_flat.grad_view(n) for n in en})
            layer = _Layer(self.layer_cfg, P, G, index=i)
            if cfg.layer_is_moe(i):
                from .moe import MoEBlock

                layer.moe = MoEBlock(cfg, i, ep_size=self.ep_size, ep_rank=self.ep_rank)
            self.layers.append(layer)
        self.anchor = torch.empty(0, device=self.device, requires_grad=True)
        self.ep_group = None
        self.zero3 = None  # parallel.zero3.ParamGatherer of a ZeRO-3 store

    # ----------------------------------------------------------- adapters
    def attach_lora(self, adapters) -> None:
        """Train LoRA adapters on a frozen base (the base store has no grads)."""
        self.lora = adapters
        for i, layer in enumerate(self.layers):
            layer.lora = adapters.layer_views(i)

    def adapters_disabled(self):
        """Context manager: forward passes see the frozen base model only (the
        LoRA adapters are detached from every layer and restored on exit) —
        the reference policy of LoRA training."""
        import contextlib

        @contextlib.contextmanager
        def _off():
            saved = [layer.lora for layer in self.layers]
            lora = self.lora
            rg = self.flat.compute.requires_grad  # the CPU path turns it on for a model without adapters
            for layer in self.layers:
                layer.lora = None
            self.lora = None
            try:
                yield
            finally:
                self.lora = lora
                for layer, l in zip(self.layers, saved):
                    layer.lora = l
                if self.flat.compute.requires_grad != rg:
                    self.flat.compute.requires_grad_(rg)

        return _off()

    def freeze(self, names: list[str]) -> None:
        """Keep the parameters ``names`` of the dense store fixed: their
        gradients are zeroed before the optimizer step (so they add nothing to
        the clip norm) and their values (bf16 and this rank's fp32 master
        part) are put back after it, so neither the update nor weight decay
        moves them (the reference sets ``requires_grad=False``,
        trainer/moe.py:275-300)."""
        flat = self.flat
        lo, hi = flat.dp_rank * flat.shard_numel, (flat.dp_rank + 1) * flat.shard_numel
        self._frozen = []
        for n in names:
            off, k = flat.offsets[n]
            a, b = max(off, lo), min(off + k, hi)
            master = flat.master[a - lo:b - lo].clone() if (flat.master is not None and a < b) else None
            if flat.sharded_compute:  # ZeRO-3: this rank keeps (and restores) only its part
                val = flat.compute[a - lo:b - lo].clone() if a < b else None
            else:
                val = flat.view(n).clone()
            self._frozen.append((n, val, (a - lo, b - lo) if a < b else None, master))

    def _check_ep_layouts(self) -> None:
        """An over-capacity expert layout invalidates the micro-batches of this
        step: report it (EPCapacityError) before the optimizer uses them."""
        for layer in self.layers:
            fe = getattr(layer.moe, "ep_fabric", None) if layer.moe is not None else None
            if fe is not None:
                fe.check()
                return

    def after_optimizer_step(self) -> None:
        for n, val, span, master in getattr(self, "_frozen", []):
            if self.flat.sharded_compute:
                if span is not None:
                    self.flat.compute[span[0]:span[1]].copy_(val)
            else:
                self.flat.view(n).copy_(val)
            if span is not None and master is not None:
                self.flat.master[span[0]:span[1]].copy_(master)

    def finalize_grads(self) -> None:
        """Cross-TP sums of gradients that each TP rank only partially owns:
        the QK-norm weights are shared by all heads, which are split.  Frozen
        parameters get zero gradients."""
        self._check_ep_layouts()
        for n, _, span, _ in getattr(self, "_frozen", []):
            if self.flat.sharded_compute:  # ZeRO-3: the reduced gradients of this rank's part
                if span is not None and self.flat.grad is not None:
                    self.flat.grad[span[0]:span[1]].zero_()
                continue
            g = self.flat.grad_view(n)
            if g is not None:
                g.zero_()
        if self.tp_size > 1 and self.flat.grad is not None:
            import torch.distributed as dist

            for layer in self.layers:
                for n in ("q_norm", "k_norm"):
                    g = layer.G.get(n)
                    if g is not None:
                        dist.all_reduce(g, group=self.tp_group)

    def attach_tp_fabric(self, fabric, capacity: int = 1 << 20):
        """Row-parallel outputs and column-parallel input gradients summed by
        the fused GEMM -> all-reduce kernels (parallel.tp_fabric) instead of
        NCCL; ``fabric`` spans the tensor-parallel group."""
        from ..parallel.tp_fabric import TPFabric

        if fabric.world != self.tp_size:
            raise ValueError("the fabric must span the tensor-parallel group")
        self.tp_fabric = TPFabric(fabric, capacity)
        return self.tp_fabric

    def attach_ep_fabric(self, fabric, capacity_rows: int = 1 << 16, max_tokens: int = 0,
                         capacity_factor: float | None = None):
        """Expert dispatch / combine over peer memory (parallel.ep_fabric) for
        every MoE layer; ``fabric`` spans the expert-parallel group.  The row
        buffers fit the worst routing of ``max_tokens`` tokens per micro-batch
        (or ``capacity_factor`` x the average copies), at least ``capacity_rows``."""
        from ..parallel.ep_fabric import FabricEP

        fe = FabricEP(fabric, self.ep_group, self.cfg.num_experts, self.cfg.hidden_size, capacity_rows,
                      k=self.cfg.num_experts_per_tok, max_tokens=max_tokens, capacity_factor=capacity_factor)
        for layer in self.layers:
            if layer.moe is not None:
                layer.moe.ep_fabric = fe
        return fe

    def set_activation_checkpointing(self, every: int | None) -> None:
        """Recompute every ``every``-th layer in backward (1: all, the
        reference's full mode with freq 1); None keeps all activations."""
        for i, layer in enumerate(self.layers):
            layer.recompute = every is not None and (i % every == 0)

    def enable_activation_offload(self, on: bool = True) -> None:
        from .layers import ActivationOffload

        off = ActivationOffload() if on else None
        for layer in self.layers:
            layer.offload = off

    @property
    def trainable(self) -> FlatParams:
        return self.lora.flat if self.lora is not None else self.flat

    # ----------------------------------------------------------- weights
    def weight(self, name: str) -> torch.Tensor:
        return self.flat.view(name)

    def grad(self, name: str) -> torch.Tensor | None:
        return self.flat.grad_view(name)

    @property
    def head_name(self) -> str:
        return "embed" if self.cfg.tie_embeddings else "lm_head"

    def head_weight(self) -> torch.Tensor:
        return self.flat.view(self.head_name)

    def head_grad(self) -> torch.Tensor | None:
        return self.flat.grad_view(self.head_name)

    # ----------------------------------------------------------- batches
    def batch_ctx(self, position_ids: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int,
                  cp=None) -> BatchCtx:
        return BatchCtx(
            pos=position_ids.to(device=self.device, dtype=torch.int32).reshape(-1).contiguous(),
            cu_seqlens=cu_seqlens.to(device=self.device, dtype=torch.int32).contiguous(),
            max_seqlen=int(max_seqlen),
            inv_freq=self.inv_freq,
            cp=cp,
        )

    # ----------------------------------------------------------- forward
    def hidden(self, input_ids: torch.Tensor, batch: BatchCtx) -> torch.Tensor:
        """Final normalised hidden states [T, H] (autograd-connected)."""
        if not input_ids.is_cuda and not self.fused_cpu and self.tp_size == 1 and batch.cp is None:
            if self.expert_flat is not None:
                raise NotImplementedError("the CPU reference path runs without expert parallelism")
            return self._hidden_cpu(input_ids.reshape(-1), batch)
        ids = input_ids.reshape(-1).contiguous()
        if self.zero3 is not None:
            self.zero3.begin_forward()
        x = EmbeddingFn.apply(ids, self.anchor, self.weight("embed"), self.grad("embed"), self.zero3)
        tpc = TPContext(self.tp_group, self.tp_rank, self.tp_size, self.tp_fabric) if self.tp_size > 1 else None
        for layer in self.layers:
            layer.batch = batch
            layer.tp = tpc
            if layer.moe is not None:
                layer.moe.ep_group = self.ep_group
            x = DecoderLayerFn.apply(x, self.anchor, layer)
        return FinalNormFn.apply(x, self.weight("norm"), self.grad("norm"), self.cfg.rms_eps)

    # CPU float32 reference path (autograd through views of flat.compute)
    def _hidden_cpu(self, ids: torch.Tensor, batch: BatchCtx) -> torch.Tensor:
        cfg = self.cfg
        flat = self.flat
        if self.lora is None and not flat.compute.requires_grad:
            flat.compute.requires_grad_(True)

        def W(n):
            if n in self.quant:
                return self.quant[n].dequantize(flat.compute.dtype)
            off, k = flat.offsets[n]
            shape = next(s.shape for s in flat.specs if s.name == n)
            return flat.compute[off : off + k].view(shape)

        lf = self.lora.flat if self.lora is not None else None
        if lf is not None and not lf.compute.requires_grad:
            lf.compute.requires_grad_(True)

        def lin(x, i, wname, target, bias=None):
            y = F.linear(x, W(f"l{i}.{wname}"), bias)
            if lf is None or f"l{i}.{target}.A" not in lf.offsets:
                return y
            lay = self.lora.layouts[target]
            r, sc = self.lora.rank, self.lora.scale
            oa, na = lf.offsets[f"l{i}.{target}.A"]
            ob, nb = lf.offsets[f"l{i}.{target}.B"]
            A = lf.compute[oa : oa + na].view(lay.kp, lay.in_dim)
            B = lf.compute[ob : ob + nb].view(lay.out_dim, lay.kp)
            parts = []
            for _, _, lo, hi, c0 in lay.parts:
                parts.append((lo, hi, sc * (x @ A[c0 : c0 + r].t()) @ B[lo:hi, c0 : c0 + r].t()))
            delta = torch.zeros_like(y)
            for lo, hi, d in parts:
                delta = delta.index_add(1, torch.arange(lo, hi), d)
            return y + delta

        T = ids.shape[0]
        nq, nk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        x = W("embed")[ids]
        for i in range(cfg.num_layers):
            p = f"l{i}."
            h = ref.rmsnorm(x, W(p + "in_norm"), cfg.rms_eps)
            qkv = lin(h, i, "qkv_w", "qkv", W(p + "qkv_b") if cfg.qkv_bias else None)
            q = qkv[:, : nq * hd].view(T, nq, hd)
            k = qkv[:, nq * hd : (nq + nk) * hd].view(T, nk, hd)
            v = qkv[:, (nq + nk) * hd :].view(T, nk, hd)
            if cfg.qk_norm:
                q = ref.rmsnorm(q, W(p + "q_norm"), cfg.rms_eps)
                k = ref.rmsnorm(k, W(p + "k_norm"), cfg.rms_eps)
            q = ref.apply_rope(q, batch.pos, batch.inv_freq)
            k = ref.apply_rope(k, batch.pos, batch.inv_freq)
            att = ref.attention(q, k, v, batch.cu_seqlens, True)
            x = x + lin(att.reshape(T, nq * hd), i, "o_w", "o")
            h2 = ref.rmsnorm(x, W(p + "post_norm"), cfg.rms_eps)
            if cfg.layer_is_moe(i):
                from .moe import moe_reference

                x = x + moe_reference(h2, W(p + "router_w"), W(p + "exp_gu_w"), W(p + "exp_down_w"), cfg)[0]
            else:
                x = x + lin(ref.swiglu(lin(h2, i, "gu_w", "gu")), i, "down_w", "down")
        return ref.rmsnorm(x, W("norm"), cfg.rms_eps)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        W = self.head_weight()
        if h.is_cuda:
            return ops.gemm(h.contiguous(), W)
        if self.flat.sharded_compute:  # the staged head (ZeRO-3)
            return h @ W.t()
        off, k = self.flat.offsets[self.head_name]
        Wv = self.flat.compute[off : off + k].view(W.shape)
        return h @ Wv.t()

    def collect_cpu_grads(self) -> None:
        """CPU path: move autograd grads of the flat buffer into flat.grad."""
        for f in (self.flat, self.lora.flat if self.lora is not None else None):
            if f is None:
                continue
            g = f.compute.grad
            if g is not None and f.grad is not None:
                f.grad.add_(g.float())
            f.compute.grad = None


def build_model(cfg: ArchConfig, device, dtype=None, dp_rank=0, dp_world=1, seed=0, init=True,
                with_grad=True, with_optimizer=True, fabric=None, lora=None, load_in_4bit: bool = False,
                lora_seed: int = 0, ep: tuple[int, int, int, int] | None = None,
                tp: tuple[int, int] | None = None, ep_fabric=None, shard_params: bool = False) -> CausalLM:
    """Build (and random-init) a model (a ``DeepseekV4Config`` builds the
    eager DeepSeek-V4 model behind the same interface).

    ``lora``: an object with ``rank``, ``alpha``, ``target_modules``, ``dropout``
    (the ``lora`` config section) -> frozen base + trainable adapters.
    ``load_in_4bit``: NF4-quantise the dense projections after init (QLoRA).
    ``ep``: (ep size, ep rank, expert-dp rank, expert-dp size) for expert
    parallelism; the expert tensors of this rank go to ``model.expert_flat``
    (in peer-visible memory of ``ep_fabric`` when given: policy refresh and
    the fused dispatch read it from the other ranks).
    ``shard_params``: ZeRO-3 — the bf16 weights are sharded over the
    ``dp_world`` ranks too (``ShardedFlatParams``); attach a
    ``parallel.zero3.ParamGatherer`` before running the model.
    """
    device = torch.device(device)
    if dtype is None:
        dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    from .deepseek_v4.config import DeepseekV4Config

    if getattr(cfg, "generic_hf", False):
        if lora is not None or load_in_4bit or ep or tp or fabric is not None or ep_fabric is not None:
            raise NotImplementedError("Hugging Face models without a native decoder train with data parallelism "
                                      "only (no LoRA / QLoRA, tensor or expert parallelism, peer fabric)")
        from .hf_generic import HFCausalLMTrainable

        return HFCausalLMTrainable(cfg, device, dtype, dp_rank, dp_world, seed, init, with_grad, with_optimizer)
    if isinstance(cfg, DeepseekV4Config):
        if lora is not None or load_in_4bit or ep or tp or fabric is not None or ep_fabric is not None:
            raise NotImplementedError("the eager DeepSeek-V4 model trains with data parallelism only "
                                      "(no LoRA / QLoRA, tensor or expert parallelism, peer fabric)")
        from .deepseek_v4.trainable import DeepseekV4Trainable

        return DeepseekV4Trainable(cfg, device, dtype, dp_rank, dp_world, seed, init, with_grad, with_optimizer)
    tp_size, tp_rank = tp or (1, 0)
    if shard_params and (lora is not None or load_in_4bit or tp_size > 1 or (ep or (1,))[0] > 1 or fabric is not None):
        raise NotImplementedError("sharded parameters (ZeRO-3) train dense or MoE models with data (and context) "
                                  "parallelism: no LoRA / NF4, tensor or expert parallelism, or fused peer optimizer")
    full_specs = param_specs(cfg)
    specs = param_specs(tp_local_cfg(cfg, tp_size)) if tp_size > 1 else full_specs
    if tp_size > 1 and (lora is not None or load_in_4bit or (ep or (1,))[0] > 1):
        raise NotImplementedError("tensor parallelism does not combine with LoRA, NF4 or expert parallelism here")
    qnames = {s.name for s in specs if load_in_4bit and s.name.split(".", 1)[-1] in QUANTIZABLE}
    frozen = lora is not None
    seed_index = {s.name: i for i, s in enumerate(full_specs)}
    tp_rows = {}
    tp_repl = []
    if tp_size > 1:
        sl = tp_slicers(cfg, tp_size, tp_rank)
        tp_rows = {s.name: sl[s.name.split(".", 1)[-1]] for s in specs if s.name.split(".", 1)[-1] in sl}
        # replicated parameters first: the gradient norm weighs [0, tp_repl_end) by 1/tp
        tp_repl = [s for s in specs if s.name not in tp_rows]
        specs = tp_repl + [s for s in specs if s.name in tp_rows]
    ep_size, ep_rank, ep_dp_rank, ep_dp_world = ep or (1, 0, 0, 1)
    expert_flat = None
    if ep_size > 1:
        if cfg.num_experts % ep_size:
            raise ValueError(f"num_experts {cfg.num_experts} is not divisible by ep {ep_size}")
        if frozen:
            raise NotImplementedError("LoRA with expert parallelism is not supported")
        el = cfg.num_experts // ep_size
        lo, hi = ep_rank * el, (ep_rank + 1) * el
        espec, rows = [], {}
        for s_ in specs:
            if is_expert_param(s_.name):
                espec.append(ParamSpec(s_.name, (el,) + tuple(s_.shape[1:]), s_.init, s_.weight_decay, s_.std))
                rows[s_.name] = (tuple(s_.shape), lo, hi)
        specs = [s_ for s_ in specs if not is_expert_param(s_.name)]
        expert_flat = FlatParams(espec, device, dtype, ep_dp_rank, ep_dp_world, with_grad, with_optimizer,
                                 alloc=ep_fabric.allocator() if ep_fabric is not None else None)
        if init:
            expert_flat.init_(seed, seed_index=seed_index, row_slices=rows)
    store = ShardedFlatParams if shard_params else FlatParams
    flat = store([s for s in specs if s.name not in qnames], device, dtype, dp_rank, dp_world,
                 with_grad and not frozen, with_optimizer and not frozen,
                 alloc=fabric.allocator() if (fabric is not None and not frozen) else None)
    if tp_repl:
        flat.set_tp_replicated([s.name for s in tp_repl], tp_size)
    quant = {}
    if init:
        flat.init_(seed, seed_index=seed_index, row_slices=tp_rows or None)
    if qnames:
        from ..ops.nf4 import quantize

        g = torch.Generator(device=device)
        for s in specs:
            if s.name not in qnames:
                continue
            tmp = torch.zeros(s.shape, device=device, dtype=torch.float32)
            if init:
                g.manual_seed(seed * 1_000_003 + seed_index[s.name])
                tmp.normal_(0.0, s.std, generator=g)
            quant[s.name] = quantize(tmp.to(dtype))
            del tmp
    model = CausalLM(cfg, flat, quant, expert_flat, (ep_size, ep_rank), tp=(tp_size, tp_rank))
    model.ep_dp_rank = ep_dp_rank
    if shard_params:
        model.fused_cpu = True  # the per-layer gathers hook the kernel-path layer functions (CPU fallbacks too)
    if frozen:
        from .lora import LoRAAdapters

        ad = LoRAAdapters(cfg, lora.rank, lora.alpha, list(lora.target_modules), device, dtype, dp_rank, dp_world,
                          dropout=getattr(lora, "dropout", 0.0), seed=lora_seed, fabric=fabric)
        model.attach_lora(ad)
    return model
