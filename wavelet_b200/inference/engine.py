"""Native batched generator (replaces the reference's vLLM engine).

* Paged KV cache: per layer ``k``/``v`` tensors [num_blocks, Hk, block_size,
  128] bf16 (head-major pages); a block manager hands out blocks, with reference counts so the
  ``n`` samples of one prompt share the prompt's full blocks (the partial last
  block is copied per sample).
* Continuous batching: sequences are admitted while blocks are free, prefilled
  as one packed batch (tcgen05 attention forward over ``cu_seqlens``), then
  advanced together one token per decode step until they hit a stop token or
  ``max_tokens``; finished sequences free their blocks and new ones join.
* Decode step: embedding -> per layer (RMSNorm, QKV GEMM, QK-norm + RoPE,
  KV append, paged decode attention, O GEMM + residual, RMSNorm, gate/up
  GEMM, SwiGLU, down GEMM + residual) -> final norm -> LM head GEMM -> fused
  sampling (Gumbel-max at temperature, processed log-prob of the sampled
  token, optional top-k / min-p / top-p support).
* Fast decode (dense models, untruncated sampling): the decode state
  (last token, position, context length, KV slot, block table, sampling
  seed) lives on the device; the host allocates KV blocks once per window of
  up to 16 steps and replays one CUDA graph per step (captured per
  batch-size bucket and split count).  A ``decode_advance`` kernel records
  the sampled token and advances the state, so a window costs one host sync.
  Stop tokens are found when the window's tokens come back; tokens sampled
  after a stop are dropped.
* Outputs match what the trainer needs: exact token ids, the processed
  log-probs at the sampling temperature, and the sampling support set when
  top-k / top-p / min-p truncate it (vLLM ``processed_logprobs`` and
  ``return_sampling_mask`` in the reference, inference/engine.py:775-944).

The engine shares the model's flat parameter store, so an in-process trainer
updates the policy in place (zero-copy policy transfer).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..utils import nvtx
from ..models.layers import _lin, _lin_rowpar
from ..models.qwen import CausalLM
from ..ops import reference as ref
from ..ops.attention import attention_fwd


def sampling_thresholds_reference(z: torch.Tensor, top_k: list[int], top_p: list[float],
                                  inv_tau: torch.Tensor) -> torch.Tensor:
    """Per-row sampling threshold in logit units (keep ``z >= thresh``): the
    k-th largest logit for top-k, and for top-p the logit at which the
    descending cumulative probability of softmax(z * inv_tau) first reaches p;
    the larger of the two, -inf where neither applies.  Sort-based float32
    oracle of the ``sample_thresholds`` kernel (and its CPU path)."""
    B = z.shape[0]
    zf = z.float()
    th = torch.full((B,), float("-inf"), device=z.device)
    for i in range(B):
        t = float("-inf")
        if top_k[i] > 0 and top_k[i] < zf.shape[1]:
            t = float(torch.topk(zf[i], top_k[i]).values[-1])
        it = float(inv_tau[i])
        if top_p[i] < 1.0 and it > 0:
            srt = torch.sort(zf[i], descending=True).values
            c = torch.softmax(srt * it, -1).cumsum(-1)
            k = int((c < top_p[i]).sum()) + 1
            t = max(t, float(srt[min(k, srt.numel()) - 1]))
        th[i] = t
    return th


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    max_tokens: int = 256
    min_tokens: int = 0
    n: int = 1
    stop_token_ids: list[int] = field(default_factory=list)
    seed: int | None = None
    return_sampling_mask: bool = False

    @property
    def truncated(self) -> bool:
        return self.top_p < 1.0 or self.top_k > 0 or self.min_p > 0.0


@dataclass
class Completion:
    prompt_index: int
    sample_index: int
    prompt_ids: list[int]
    token_ids: list[int]
    logprobs: list[float]
    finish_reason: str
    sampling_mask: list[list[int]] | None = None


@dataclass
class _Seq:
    pid: int
    sidx: int
    prompt: list[int]
    params: SamplingParams
    blocks: list[int]
    length: int  # tokens in cache
    out: list[int] = field(default_factory=list)
    lps: list[float] = field(default_factory=list)
    masks: list[list[int]] | None = None
    done: str | None = None
    row_id: int = 0


class BlockManager:
    def __init__(self, num_blocks: int):
        self.free = list(range(num_blocks - 1, -1, -1))
        self.ref = [0] * num_blocks

    def alloc(self) -> int:
        if not self.free:
            raise MemoryError("KV cache out of blocks")
        b = self.free.pop()
        self.ref[b] = 1
        return b

    def share(self, b: int) -> int:
        self.ref[b] += 1
        return b

    def release(self, blocks: list[int]) -> None:
        for b in blocks:
            self.ref[b] -= 1
            if self.ref[b] == 0:
                self.free.append(b)

    @property
    def num_free(self) -> int:
        return len(self.free)


class Generator:
    def __init__(self, model: CausalLM, *, max_num_seqs: int = 512, max_model_len: int = 4096,
                 kv_cache_bytes: int | None = None, gpu_memory_utilization: float | None = None,
                 block_size: int = 64, decode_splits: int | None = None, cuda_graphs: bool = True,
                 window: int = 16):
        self.m = model
        cfg = model.cfg
        self.cfg = cfg
        # tensor parallelism (Megatron split of a TP-trained model): this rank
        # runs its heads and FFN columns, row-parallel outputs are summed over
        # the TP group; the LM head and norms are replicated, so every rank
        # samples the same tokens from identical logits and a shared seed
        self.tp = getattr(model, "tp_size", 1)
        self.lc = getattr(model, "layer_cfg", cfg)  # this rank's head counts
        if self.tp > 1 and any(layer.moe is not None for layer in model.layers):
            raise NotImplementedError("tensor-parallel generation of MoE models is not supported")
        self.dev = model.device
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.max_model_len = max_model_len
        per_block = 2 * cfg.num_layers * block_size * self.lc.num_kv_heads * cfg.head_dim * 2
        if kv_cache_bytes is None:
            if self.dev.type == "cuda":
                free, total = torch.cuda.mem_get_info(self.dev)
                frac = gpu_memory_utilization if gpu_memory_utilization is not None else 0.35
                kv_cache_bytes = int(min(free * 0.9, total * frac))
            else:
                kv_cache_bytes = 64 * per_block
        self.num_blocks = max(4, kv_cache_bytes // per_block)
        # head-major pages: one head's tokens of a block are contiguous (decode
        # attention streams 8 KB runs per head instead of 256-byte pieces)
        shape = (self.num_blocks, self.lc.num_kv_heads, block_size, cfg.head_dim)
        dt = model.flat.compute_dtype
        self.k_cache = [torch.empty(shape, device=self.dev, dtype=dt) for _ in range(cfg.num_layers)]
        self.v_cache = [torch.empty(shape, device=self.dev, dtype=dt) for _ in range(cfg.num_layers)]
        self.bm = BlockManager(self.num_blocks)
        self.sink_block = self.bm.alloc()  # KV writes of padded graph rows land here
        self.max_blocks_per_seq = (max_model_len + block_size - 1) // block_size + 1
        self.decode_splits = decode_splits
        self.stats: dict[str, float] = {}
        self._moe = [layer.moe for layer in model.layers]
        self.window = window
        # graphs replay fixed launches: TP collectives (host-side epochs, NCCL) stay eager
        self.use_graphs = (cuda_graphs and self.dev.type == "cuda" and not any(self._moe) and not model.quant
                           and self.tp == 1)
        self._bufs: dict[int, dict[str, torch.Tensor]] = {}
        self._graphs: dict[tuple[int, int], torch.cuda.CUDAGraph] = {}
        self._graph_kernels: dict[tuple[int, int], int] = {}
        self._graph_pool = None

    # ------------------------------------------------------------ utilities
    def release_cache(self) -> None:
        """Free the KV cache memory (``sleep``); ``restore_cache`` re-allocates it."""
        self._cache_shape = self.k_cache[0].shape if self.k_cache else None
        self.k_cache = []
        self.v_cache = []
        if self.dev.type == "cuda":
            torch.cuda.empty_cache()

    def restore_cache(self) -> None:
        if self.k_cache or getattr(self, "_cache_shape", None) is None:
            return
        dt = self.m.flat.compute_dtype
        self.k_cache = [torch.empty(self._cache_shape, device=self.dev, dtype=dt) for _ in range(self.cfg.num_layers)]
        self.v_cache = [torch.empty(self._cache_shape, device=self.dev, dtype=dt) for _ in range(self.cfg.num_layers)]
        self.bm = BlockManager(self.num_blocks)

    def kv_usage(self) -> float:
        return 1.0 - self.bm.num_free / self.num_blocks

    def _slots(self, seqs: list[_Seq], positions: list[list[int]]) -> torch.Tensor:
        out = []
        for s, ps in zip(seqs, positions):
            for p in ps:
                out.append(s.blocks[p // self.block_size] * self.block_size + p % self.block_size)
        return torch.tensor(out, dtype=torch.int32, device=self.dev)

    def _ensure_blocks(self, s: _Seq, upto: int) -> None:
        while len(s.blocks) * self.block_size < upto:
            s.blocks.append(self.bm.alloc())

    # -------------------------------------------------------------- forward
    def _layers_forward(self, x, pos, slots, attn_fn):
        cfg = self.cfg
        nq, nk, hd = self.lc.num_heads, self.lc.num_kv_heads, cfg.head_dim
        T = x.shape[0]
        tpc = None
        if self.tp > 1:
            from ..models.qwen import TPContext

            tpc = TPContext(self.m.tp_group, self.m.tp_rank, self.tp, self.m.tp_fabric)
        for li, layer in enumerate(self.m.layers):
            P = layer.P
            lora = layer.lora or {}
            h, _, _ = ops.rmsnorm_fwd(x, P["in_norm"], cfg.rms_eps)
            qkv, _ = _lin(h, P["qkv_w"], lora.get("qkv"), bias=P.get("qkv_b"))
            ops.qk_norm_rope_(qkv, nq, nk, pos, self.m.inv_freq, P.get("q_norm"), P.get("k_norm"), cfg.rms_eps)
            q = qkv[:, : nq * hd].view(T, nq, hd)
            k = qkv[:, nq * hd : (nq + nk) * hd].view(T, nk, hd)
            v = qkv[:, (nq + nk) * hd :].view(T, nk, hd)
            if x.is_cuda:
                ops.ext().kv_append(k, v, self.k_cache[li], self.v_cache[li], slots)
            else:
                sl = slots.long()
                blk, off = sl // self.block_size, sl % self.block_size
                self.k_cache[li][blk, :, off] = k
                self.v_cache[li][blk, :, off] = v
            att = attn_fn(li, q, k, v)
            x, _ = _lin_rowpar(att.reshape(T, nq * hd), P["o_w"], lora.get("o"), x, tpc)
            if layer.moe is not None:
                h2, _, _ = ops.rmsnorm_fwd(x, P["post_norm"], cfg.rms_eps)
                x = layer.moe.infer(h2, x, P)
            else:
                h2, _, _ = ops.rmsnorm_fwd(x, P["post_norm"], cfg.rms_eps)
                a = ops.swiglu_fwd(_lin(h2, P["gu_w"], lora.get("gu"))[0])
                x, _ = _lin_rowpar(a, P["down_w"], lora.get("down"), x, tpc)
        hf, _, _ = ops.rmsnorm_fwd(x, self.m.weight("norm"), cfg.rms_eps)
        return hf

    @torch.no_grad()
    def _prefill(self, seqs: list[_Seq]) -> torch.Tensor:
        """Packed prefill of the prompts; returns final hidden of each last prompt token."""
        ids = torch.tensor([t for s in seqs for t in s.prompt], device=self.dev, dtype=torch.long)
        lens = [len(s.prompt) for s in seqs]
        cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
        cu[1:] = torch.tensor(lens).cumsum(0)
        pos = torch.cat([torch.arange(L, dtype=torch.int32) for L in lens]).to(self.dev)
        slots = self._slots(seqs, [list(range(L)) for L in lens])
        cu_d = cu.to(self.dev)
        maxlen = max(lens)
        x = ops.embedding_fwd(self.m.weight("embed"), ids)

        def attn(li, q, k, v):
            o, _ = attention_fwd(q, k, v, cu_d, maxlen, True)
            return o

        hf = self._layers_forward(x, pos, slots, attn)
        last = (cu[1:] - 1).to(self.dev).long()
        return hf[last]

    @torch.no_grad()
    def _decode(self, seqs: list[_Seq]) -> torch.Tensor:
        B = len(seqs)
        ids = torch.tensor([s.out[-1] if s.out else s.prompt[-1] for s in seqs], device=self.dev, dtype=torch.long)
        pos_l = [s.length for s in seqs]
        for s in seqs:
            self._ensure_blocks(s, s.length + 1)
        slots = self._slots(seqs, [[p] for p in pos_l])
        pos = torch.tensor(pos_l, dtype=torch.int32, device=self.dev)
        ctx = torch.tensor([p + 1 for p in pos_l], dtype=torch.int32, device=self.dev)
        bt = torch.zeros(B, self.max_blocks_per_seq, dtype=torch.int32)
        for i, s in enumerate(seqs):
            bt[i, : len(s.blocks)] = torch.tensor(s.blocks, dtype=torch.int32)
        bt = bt.to(self.dev)
        max_ctx = max(pos_l) + 1
        splits = self.decode_splits or self._splits(B, max_ctx)
        x = ops.embedding_fwd(self.m.weight("embed"), ids)
        scale = 1.0 / math.sqrt(self.cfg.head_dim)

        def attn(li, q, k, v):
            if not q.is_cuda:
                return self._decode_attn_ref(li, q, bt, ctx, scale)
            out = torch.empty(q.shape, device=self.dev, dtype=q.dtype)
            ops.ext().decode_attention(q, self.k_cache[li], self.v_cache[li], bt, ctx, out, splits, scale)
            return out

        return self._layers_forward(x, pos, slots, attn)

    def _decode_attn_ref(self, li, q, bt, ctx, scale):
        """Dense attention over the gathered paged KV (CPU path and oracle)."""
        B, Hq, D = q.shape
        Hk = self.lc.num_kv_heads
        out = torch.empty_like(q)
        for i in range(B):
            L = int(ctx[i])
            nb = (L + self.block_size - 1) // self.block_size
            blocks = bt[i, :nb].long()
            kk = self.k_cache[li][blocks].transpose(1, 2).reshape(-1, Hk, D)[:L].float()
            vv = self.v_cache[li][blocks].transpose(1, 2).reshape(-1, Hk, D)[:L].float()
            kk = kk.repeat_interleave(Hq // Hk, 1)
            vv = vv.repeat_interleave(Hq // Hk, 1)
            sc = torch.einsum("hd,lhd->hl", q[i].float(), kk) * scale
            out[i] = torch.einsum("hl,lhd->hd", sc.softmax(-1), vv).to(q.dtype)
        return out

    def _sample(self, hf: torch.Tensor, seqs: list[_Seq], step_seed: int):
        z = self.m.logits(hf)  # [B, V] bf16
        B = z.shape[0]
        inv_tau = torch.tensor([(1.0 / s.params.temperature) if s.params.temperature > 0 else 0.0 for s in seqs],
                               device=self.dev, dtype=torch.float32)
        thresh = None
        need_k = any(s.params.top_k > 0 for s in seqs)
        need_p = any(s.params.top_p < 1.0 for s in seqs)
        if (need_k or need_p) and z.is_cuda:
            # device radix select over the bf16 logits: no sort, no per-row host work
            thresh = torch.empty(B, device=self.dev, dtype=torch.float32)
            tk = torch.tensor([s.params.top_k for s in seqs], dtype=torch.int32, device=self.dev) if need_k else None
            tp = torch.tensor([s.params.top_p for s in seqs], dtype=torch.float32, device=self.dev) if need_p else None
            ops.ext().sample_thresholds(z, tk, tp, inv_tau, thresh)
        elif need_k or need_p:
            thresh = sampling_thresholds_reference(z, [s.params.top_k for s in seqs],
                                                   [s.params.top_p for s in seqs], inv_tau)
        min_p = max((s.params.min_p for s in seqs), default=0.0)
        tok = torch.empty(B, dtype=torch.long, device=self.dev)
        lp = torch.empty(B, dtype=torch.float32, device=self.dev)
        if z.is_cuda:
            row_ids = torch.tensor([s.row_id for s in seqs], dtype=torch.long, device=self.dev)
            ops.ext().sample_tokens(z, inv_tau, thresh, float(min_p), int(step_seed), row_ids, tok, lp)
        else:
            # temperature 0 (inv_tau 0) is greedy at scale 1, as in the sampling kernel
            greedy = inv_tau <= 0
            zt = z.float() * torch.where(greedy, torch.ones_like(inv_tau), inv_tau)[:, None]
            if thresh is not None:
                zt = zt.masked_fill(z.float() < thresh[:, None], float("-inf"))
            g = torch.Generator().manual_seed(int(step_seed))
            probs = torch.softmax(zt, -1)
            tok = torch.multinomial(probs, 1, generator=g)[:, 0]
            tok = torch.where(greedy, zt.argmax(-1), tok)
            lp = torch.log_softmax(zt, -1).gather(1, tok[:, None])[:, 0]
        masks = None
        if any(s.params.truncated and s.params.return_sampling_mask for s in seqs):
            keep = torch.ones_like(z, dtype=torch.bool)
            if thresh is not None:
                keep &= z.float() >= thresh[:, None]
            if min_p > 0:
                zt = z.float() * inv_tau[:, None]
                keep &= zt >= (zt.max(-1, keepdim=True).values + math.log(min_p))
            # one device -> host transfer for every row's kept token ids
            nz = keep.nonzero().cpu()
            counts = keep.sum(-1).cpu().tolist()
            cols = nz[:, 1].tolist()
            masks, off = [], 0
            for i in range(B):
                masks.append(cols[off:off + counts[i]] if seqs[i].params.return_sampling_mask else None)
                off += counts[i]
        return tok, lp, masks

    # -------------------------------------------------------------- driver
    def generate(self, prompts: list[list[int]], params: SamplingParams) -> list[Completion]:
        """Generate ``params.n`` completions for every prompt."""
        t0 = time.perf_counter()
        base_seed = params.seed if params.seed is not None else int(time.time_ns() & 0x7FFFFFFF)
        if self.tp > 1:  # one seed for the TP group: identical logits then sample identical tokens
            import torch.distributed as dist

            t = torch.tensor([base_seed], dtype=torch.long, device=self.dev)
            dist.broadcast(t, src=dist.get_global_rank(self.m.tp_group, 0), group=self.m.tp_group)
            base_seed = int(t.item())
        pending: list[tuple[int, list[int]]] = list(enumerate(prompts))
        active: list[_Seq] = []
        finished: list[_Seq] = []
        gen_tokens = 0
        step = 0
        row_counter = 0
        n_windows = n_eager = n_prefill = 0
        captures0 = len(self._graphs)
        while pending or active:
            # admit whole prompt groups while capacity allows
            admit: list[_Seq] = []
            while pending and len(active) + len(admit) + params.n <= self.max_num_seqs:
                pid, pr = pending[0]
                # the group shares the prompt's full blocks; each sample owns the rest
                shared = len(pr) // self.block_size
                total = (len(pr) + params.max_tokens + self.block_size - 1) // self.block_size
                need = shared + params.n * (total - shared)
                if need > self.bm.num_free and (active or admit):
                    break
                pending.pop(0)
                if len(pr) + params.max_tokens > self.max_model_len:
                    raise ValueError(f"prompt {pid} of {len(pr)} tokens + max_tokens exceeds max_model_len={self.max_model_len}")
                first = _Seq(pid, 0, list(pr), params, [], 0, row_id=row_counter)
                row_counter += 1
                self._ensure_blocks(first, len(pr))
                admit.append(first)
            if admit:
                n_prefill += 1
                hf = self._prefill(admit)
                for s in admit:
                    s.length = len(s.prompt)
                groups = []
                for s in admit:
                    grp = [s]
                    full = len(s.prompt) // self.block_size
                    for j in range(1, params.n):
                        c = _Seq(s.pid, j, s.prompt, params, [self.bm.share(b) for b in s.blocks[:full]], s.length,
                                 row_id=row_counter)
                        row_counter += 1
                        if full < len(s.blocks):  # copy the partial block
                            nb = self.bm.alloc()
                            for li in range(self.cfg.num_layers):
                                self.k_cache[li][nb].copy_(self.k_cache[li][s.blocks[full]])
                                self.v_cache[li][nb].copy_(self.v_cache[li][s.blocks[full]])
                            c.blocks.append(nb)
                        grp.append(c)
                    groups.append(grp)
                hf_rep = torch.cat([hf[i : i + 1].expand(len(g), -1) for i, g in enumerate(groups)])
                new = [c for g in groups for c in g]
                tok, lp, masks = self._sample(hf_rep, new, base_seed * 1000003 + step)
                self._append(new, tok, lp, masks)
                active += new
                gen_tokens += len(new)
            elif active and self._fast_ok(active):
                with nvtx.range("generate.decode_window"):
                    n = self._decode_window(active, base_seed * 1000003 + step)
                gen_tokens += n
                step += self._last_window - 1
                n_windows += 1
            elif active:
                n_eager += 1
                hf = self._decode(active)
                for s in active:
                    s.length += 1
                tok, lp, masks = self._sample(hf, active, base_seed * 1000003 + step)
                self._append(active, tok, lp, masks)
                gen_tokens += len(active)
            step += 1
            still = []
            for s in active:
                if s.done:
                    self.bm.release(s.blocks)
                    s.blocks = []
                    finished.append(s)
                else:
                    still.append(s)
            active = still
        dt = time.perf_counter() - t0
        self.stats = {"generated_tokens": float(gen_tokens), "seconds": dt, "tokens_per_second": gen_tokens / max(dt, 1e-9),
                      "decode_steps": float(step), "decode_windows": float(n_windows), "eager_steps": float(n_eager),
                      "prefills": float(n_prefill), "graph_captures": float(len(self._graphs) - captures0)}
        finished.sort(key=lambda s: (s.pid, s.sidx))
        return [Completion(s.pid, s.sidx, s.prompt, s.out, s.lps, s.done or "length", s.masks) for s in finished]

    def _splits(self, B: int, max_ctx: int) -> int:
        """Split the context only when (sequences x kv heads) CTAs cannot fill
        the GPU (~3 resident per SM); each split keeps >= 2 stages of 32 tokens.
        Powers of two keep the number of captured graphs small."""
        ctas = B * self.lc.num_kv_heads
        want = max(1, -(-3 * 148 // max(1, ctas)))
        cap = max(1, max_ctx // 64)
        sp = max(1, min(16, want, cap))
        return 1 << (sp.bit_length() - 1)

    # ------------------------------------------------------- fast decode
    def _fast_ok(self, seqs: list[_Seq]) -> bool:
        if self.dev.type != "cuda" or len(seqs) > 1024:
            return False
        # untruncated sampling has the whole vocabulary as its support: no mask to record
        return all(not s.params.truncated for s in seqs)

    @staticmethod
    def _bucket(B: int) -> int:
        return max(32, (B + 31) // 32 * 32) if B <= 256 else (B + 127) // 128 * 128

    def _buffers(self, Bb: int) -> dict[str, torch.Tensor]:
        b = self._bufs.get(Bb)
        if b is None:
            d, W = self.dev, self.window
            b = dict(ids=torch.zeros(Bb, dtype=torch.long, device=d), pos=torch.zeros(Bb, dtype=torch.int32, device=d),
                     ctx=torch.ones(Bb, dtype=torch.int32, device=d), slots=torch.zeros(Bb, dtype=torch.int32, device=d),
                     bt=torch.zeros(Bb, self.max_blocks_per_seq, dtype=torch.int32, device=d),
                     inv_tau=torch.ones(Bb, dtype=torch.float32, device=d),
                     row_ids=torch.zeros(Bb, dtype=torch.long, device=d),
                     seed=torch.zeros(1, dtype=torch.long, device=d), step=torch.zeros(1, dtype=torch.int32, device=d),
                     win_tok=torch.zeros(Bb, W, dtype=torch.long, device=d),
                     win_lp=torch.zeros(Bb, W, dtype=torch.float32, device=d),
                     tok=torch.zeros(Bb, dtype=torch.long, device=d), lp=torch.zeros(Bb, dtype=torch.float32, device=d))
            self._bufs[Bb] = b
        return b

    def _step_on(self, b: dict[str, torch.Tensor], splits: int) -> None:
        """One decode step entirely on device buffers (graph-capturable)."""
        scale = 1.0 / math.sqrt(self.cfg.head_dim)
        x = ops.embedding_fwd(self.m.weight("embed"), b["ids"])

        def attn(li, q, k, v):
            out = torch.empty(q.shape, device=self.dev, dtype=q.dtype)
            ops.ext().decode_attention(q, self.k_cache[li], self.v_cache[li], b["bt"], b["ctx"], out, splits, scale)
            return out

        hf = self._layers_forward(x, b["pos"], b["slots"], attn)
        z = self.m.logits(hf)
        ext = ops.ext()
        ext.sample_tokens(z, b["inv_tau"], None, 0.0, 0, b["row_ids"], b["tok"], b["lp"], b["seed"])
        ext.decode_advance(b["tok"], b["lp"], b["ids"], b["pos"], b["ctx"], b["slots"], b["bt"], self.block_size,
                           b["win_tok"], b["win_lp"], b["step"], b["seed"])

    def _run_step(self, Bb: int, splits: int) -> None:
        b = self._buffers(Bb)
        if not self.use_graphs:
            self._step_on(b, splits)
            return
        key = (Bb, splits)
        g = self._graphs.get(key)
        if g is None:
            # capture on a snapshot of the state, then restore it: warm-up and
            # capture both execute the step once
            saved = {k: v.clone() for k, v in b.items()}
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(s):
                self._step_on(b, splits)
            torch.cuda.current_stream(self.dev).wait_stream(s)
            for k, v in saved.items():
                b[k].copy_(v)
            g = torch.cuda.CUDAGraph()
            if self._graph_pool is None:
                self._graph_pool = torch.cuda.graph_pool_handle()
            m = ops.ext()
            n0 = m.launch_count()
            with torch.cuda.graph(g, pool=self._graph_pool):
                self._step_on(b, splits)
            self._graph_kernels[key] = m.launch_count() - n0  # library kernels inside the graph
            for k, v in saved.items():
                b[k].copy_(v)
            self._graphs[key] = g
        g.replay()
        ops.ext().note_launches(self._graph_kernels.get(key, 0))  # replayed kernels count as launches

    @torch.no_grad()
    def _decode_window(self, seqs: list[_Seq], seed: int) -> int:
        B = len(seqs)
        n = min(self.window, max(1, min(s.params.max_tokens - len(s.out) for s in seqs)))
        self._last_window = n
        for s in seqs:  # KV slots for positions length .. length + n - 1
            self._ensure_blocks(s, s.length + n)
        Bb = self._bucket(B)
        b = self._buffers(Bb)
        bs = self.block_size
        bt = np.full((Bb, self.max_blocks_per_seq), self.sink_block, dtype=np.int32)
        pos = np.zeros(Bb, dtype=np.int32)
        ids = np.zeros(Bb, dtype=np.int64)
        inv = np.ones(Bb, dtype=np.float32)
        rid = np.zeros(Bb, dtype=np.int64)
        for i, s in enumerate(seqs):
            bt[i, : len(s.blocks)] = s.blocks
            pos[i] = s.length
            ids[i] = s.out[-1] if s.out else s.prompt[-1]
            t = s.params.temperature
            inv[i] = (1.0 / t) if t > 0 else 0.0
            rid[i] = s.row_id
        slots = bt[np.arange(Bb), np.minimum(pos // bs, self.max_blocks_per_seq - 1)] * bs + pos % bs
        host = {"bt": bt, "pos": pos, "ctx": pos + 1, "slots": slots.astype(np.int32), "ids": ids, "inv_tau": inv,
                "row_ids": rid}
        for k, v in host.items():
            b[k].copy_(torch.from_numpy(v), non_blocking=False)
        b["step"].zero_()
        b["seed"].fill_(seed)
        max_ctx = int(pos[:B].max()) + n + 1
        splits = self.decode_splits or self._splits(B, max_ctx)
        for _ in range(n):
            self._run_step(Bb, splits)
        toks = b["win_tok"][:B, :n].cpu().tolist()
        lps = b["win_lp"][:B, :n].cpu().tolist()
        produced = 0
        for i, s in enumerate(seqs):
            for j in range(n):
                s.out.append(int(toks[i][j]))
                s.lps.append(float(lps[i][j]))
                s.length += 1
                produced += 1
                k = len(s.out)
                if k >= s.params.max_tokens:
                    s.done = "length"
                elif k >= s.params.min_tokens and s.out[-1] in s.params.stop_token_ids:
                    s.done = "stop"
                if s.done:
                    break
        return produced

    def _append(self, seqs: list[_Seq], tok: torch.Tensor, lp: torch.Tensor, masks) -> None:
        tl = tok.tolist()
        ll = lp.tolist()
        for i, s in enumerate(seqs):
            t = int(tl[i])
            s.out.append(t)
            s.lps.append(float(ll[i]))
            if masks is not None and masks[i] is not None:
                if s.masks is None:
                    s.masks = []
                s.masks.append(masks[i])
            n = len(s.out)
            if n >= s.params.max_tokens:
                s.done = "length"
            elif n >= s.params.min_tokens and t in s.params.stop_token_ids:
                s.done = "stop"
