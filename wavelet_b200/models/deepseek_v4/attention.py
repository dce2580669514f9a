"""DeepSeek-V4 attention over packed documents (reference
trainer/models/deepseek_v4/attention.py).

Every layer attends, per query, over one gathered key list:

* the local window: the last ``sliding_window`` tokens of the query's own
  document, itself included;
* for compressed layers, compressed entries: each pools ``rate`` consecutive
  tokens of a document into one ``head_dim`` vector (softmax gate over the
  window, RMS-normalised, rotated at the window's first position).  An entry
  becomes readable once the query reaches its last source token.  HCA layers
  read every readable entry of the document; CSA layers (overlapping windows
  of two series, stride ``rate``) read the ``index_topk`` entries chosen by a
  no-grad indexer that scores entries with fp8-rounded query/key products.

Keys are shared by all heads (one ``head_dim`` vector per token, MQA) and
double as values; since they carry RoPE, the output is rotated back by the
query's angle.  A learned per-head sink logit joins the softmax with a zero
value.  The output projection is grouped: ``o_groups`` blocks of heads each
map to ``o_lora_rank`` channels, then one linear mixes them.

All tensors here are one packed row (``[T, ...]``, no batch axis); documents
never see each other, and positions restart at each document.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .config import DeepseekV4Config
from .layers import DualRotary, RMSNorm, rms_unweighted, rope_interleaved

IGNORE = -1


@dataclass(frozen=True)
class EntryLayout:
    tokens: Tensor      # [E, rate] packed token index of every source token
    doc: Tensor         # [E] document of each entry
    local: Tensor       # [E] entry index inside its document
    doc_first: Tensor   # [n_docs] index of each document's first entry
    max_per_doc: int


@dataclass(frozen=True)
class PackedLayout:
    positions: Tensor   # [T] position inside the token's document
    doc: Tensor         # [T] document of each token
    rope: dict          # kind -> (cos, sin) [T, rope/2]
    window: Tensor      # [T, sliding_window] token indices, IGNORE for empty slots
    entries: dict       # rate -> EntryLayout

    @staticmethod
    def build(rotary: DualRotary, seq_lens: Tensor, dtype: torch.dtype, device) -> "PackedLayout":
        cfg = rotary.config
        lens = seq_lens.to(device=device, dtype=torch.int64)
        starts = torch.cumsum(lens, 0) - lens
        T = int(lens.sum())
        tok = torch.arange(T, device=device)
        doc = torch.repeat_interleave(torch.arange(lens.numel(), device=device), lens)
        pos = tok - starts[doc]
        rope = {k: rotary(pos, k, dtype) for k in rotary.kinds}
        W = cfg.sliding_window
        first = torch.maximum(tok - pos, tok - W + 1)
        slots = first[:, None] + torch.arange(W, device=device)[None, :]
        window = torch.where(slots <= tok[:, None], slots, torch.full_like(slots, IGNORE))
        rates = {cfg.compress_rates[t] for t in cfg.layer_types if t != "sliding_attention"}
        entries = {}
        for r in rates:
            per_doc = lens // r
            edoc = torch.repeat_interleave(torch.arange(lens.numel(), device=device), per_doc)
            doc_first = torch.cumsum(per_doc, 0) - per_doc
            local = torch.arange(int(per_doc.sum()), device=device) - doc_first[edoc]
            tokens = starts[edoc, None] + local[:, None] * r + torch.arange(r, device=device)[None, :]
            entries[r] = EntryLayout(tokens, edoc, local, doc_first, int(per_doc.max()) if per_doc.numel() else 0)
        return PackedLayout(pos, doc, rope, window, entries)


def fp8_round(x: Tensor) -> Tensor:
    """Round-trip through float8 e4m3 with a power-of-two scale per row."""
    amax = x.float().abs().amax(-1, keepdim=True).clamp_min(1e-10)
    scale = torch.exp2(torch.ceil(torch.log2(amax / 448.0)))
    return (x.float() / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float() * scale


class GroupedLinear(nn.Linear):
    """Block-diagonal linear: input [..., g, in/g] -> [..., g, out/g]; the
    weight is stored as an ordinary [out, in/g] matrix (group-major rows)."""

    def __init__(self, in_per_group: int, out_features: int, groups: int):
        super().__init__(in_per_group, out_features, bias=False)
        self.groups = groups

    def forward(self, x: Tensor) -> Tensor:
        w = self.weight.view(self.groups, -1, self.weight.shape[-1])
        return torch.einsum("...gi,goi->...go", x, w)


class Compressor(nn.Module):
    """Softmax-gated pooling of ``rate`` tokens into one entry.  With
    ``series == 2`` the first ``head_dim`` channels of the projections form a
    series read from the previous entry's tokens (windows overlap by one
    stride; a document's first entry has none)."""

    def __init__(self, config: DeepseekV4Config, head_dim: int, rate: int, series: int):
        super().__init__()
        self.rate, self.head_dim, self.series = rate, head_dim, series
        self.kv_proj = nn.Linear(config.hidden_size, series * head_dim, bias=False)
        self.gate_proj = nn.Linear(config.hidden_size, series * head_dim, bias=False)
        self.position_bias = nn.Parameter(torch.zeros(rate, series * head_dim))
        self.kv_norm = RMSNorm(head_dim, config.rms_norm_eps)
        self.rotary = DualRotary(config)

    def entries(self, h: Tensor, layout: PackedLayout) -> Tensor:
        """h [T, H] -> entries [E, head_dim]."""
        el = layout.entries[self.rate]
        d = self.head_dim
        kv = self.kv_proj(h)[el.tokens]                        # [E, rate, series*d]
        gate = self.gate_proj(h)[el.tokens] + self.position_bias
        if self.series == 2:
            prev = (torch.arange(kv.shape[0], device=h.device) - 1).clamp_min(0)
            first = (el.local == 0)[:, None, None]
            kv = torch.cat([kv[prev, :, :d].masked_fill(first, 0.0), kv[..., d:]], dim=1)
            gate = torch.cat([gate[prev, :, :d].masked_fill(first, float("-inf")), gate[..., d:]], dim=1)
        w = torch.softmax(gate.float(), dim=1).to(kv.dtype)
        pooled = self.kv_norm((kv * w).sum(1))
        cos, sin = self.rotary(el.local * self.rate, "compress", pooled.dtype)
        return rope_interleaved(pooled, cos, sin)

    def readable(self, layout: PackedLayout) -> Tensor:
        """Entries of its own document a query may read: (pos + 1) // rate."""
        return (layout.positions + 1) // self.rate


class Indexer(nn.Module):
    """No-grad top-k selection of compressed entries for CSA layers."""

    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        self.heads, self.head_dim, self.topk = config.index_n_heads, config.index_head_dim, config.index_topk
        self.compressor = Compressor(config, config.index_head_dim,
                                     config.compress_rates["compressed_sparse_attention"], 2)
        self.q_b_proj = nn.Linear(config.q_lora_rank, self.heads * self.head_dim, bias=False)
        self.weights_proj = nn.Linear(config.hidden_size, self.heads, bias=False)
        for p in self.parameters():
            p.requires_grad_(False)

    @torch.no_grad()
    def forward(self, h: Tensor, q_res: Tensor, layout: PackedLayout) -> Tensor:
        """[T, topk] entry indices (IGNORE for unused picks)."""
        keys = self.compressor.entries(h, layout)                       # [E, dI]
        T, E = h.shape[0], keys.shape[0]
        out = torch.full((T, self.topk), IGNORE, dtype=torch.long, device=h.device)
        if E == 0:
            return out
        cos, sin = layout.rope["compress"]
        q = rope_interleaved(self.q_b_proj(q_res).view(T, self.heads, self.head_dim), cos[:, None], sin[:, None])
        w = self.weights_proj(h).float()                                 # [T, heads]
        score = (torch.einsum("thd,ed->the", fp8_round(q), fp8_round(keys)).relu() * w[..., None]).sum(1)
        el = layout.entries[self.compressor.rate]
        lo = el.doc_first[layout.doc]
        hi = lo + self.compressor.readable(layout)
        e = torch.arange(E, device=h.device)
        ok = (e[None] >= lo[:, None]) & (e[None] < hi[:, None])
        k = min(self.topk, E)
        pick = score.masked_fill(~ok, float("-inf")).topk(k, dim=-1).indices
        valid = (pick >= lo[:, None]) & (pick < hi[:, None])
        out[:, :k] = torch.where(valid, pick, torch.full_like(pick, IGNORE))
        return out


class CSACompressor(Compressor):
    def __init__(self, config: DeepseekV4Config):
        super().__init__(config, config.head_dim, config.compress_rates["compressed_sparse_attention"], 2)
        self.indexer = Indexer(config)

    def forward(self, h: Tensor, q_res: Tensor, layout: PackedLayout) -> tuple[Tensor, Tensor]:
        return self.entries(h, layout), self.indexer(h, q_res, layout)


class HCACompressor(Compressor):
    def __init__(self, config: DeepseekV4Config):
        super().__init__(config, config.head_dim, config.compress_rates["heavily_compressed_attention"], 1)

    def forward(self, h: Tensor, q_res: Tensor, layout: PackedLayout) -> tuple[Tensor, Tensor]:
        el = layout.entries[self.rate]
        n = self.readable(layout)[:, None]
        j = torch.arange(el.max_per_doc, device=h.device)[None, :]
        picks = torch.where(j < n, el.doc_first[layout.doc][:, None] + j, torch.full_like(j, IGNORE))
        return self.entries(h, layout), picks


def gathered_attention(q: Tensor, keys: Tensor, slots: Tensor, sinks: Tensor, scale: float) -> Tensor:
    """q [T, h, d], keys [N, d], slots [T, S] (IGNORE = absent) -> [T, h, d]."""
    absent = slots < 0
    g = keys[slots.clamp_min(0)].masked_fill(absent[..., None], 0.0)  # [T, S, d]
    s = torch.einsum("thd,tsd->ths", q.float(), g.float()) * scale
    s = s.masked_fill(absent[:, None, :], float("-inf"))
    s = torch.cat([s, sinks.float()[None, :, None].expand(s.shape[0], -1, 1)], dim=-1)
    p = torch.softmax(s, dim=-1)[..., :-1].to(g.dtype)
    return torch.einsum("ths,tsd->thd", p, g)


class Attention(nn.Module):
    def __init__(self, config: DeepseekV4Config, layer_idx: int):
        super().__init__()
        if config.attention_dropout:
            raise ValueError("DeepSeek-V4 eager attention requires attention_dropout = 0")
        self.config = config
        self.kind = config.layer_types[layer_idx]
        self.rope_kind = "main" if self.kind == "sliding_attention" else "compress"
        self.heads, self.head_dim = config.num_attention_heads, config.head_dim
        self.q_a_proj = nn.Linear(config.hidden_size, config.q_lora_rank, bias=False)
        self.q_a_norm = RMSNorm(config.q_lora_rank, config.rms_norm_eps)
        self.q_b_proj = nn.Linear(config.q_lora_rank, self.heads * self.head_dim, bias=False)
        self.kv_proj = nn.Linear(config.hidden_size, self.head_dim, bias=False)
        self.kv_norm = RMSNorm(self.head_dim, config.rms_norm_eps)
        g = config.o_groups
        self.o_a_proj = GroupedLinear(self.heads * self.head_dim // g, g * config.o_lora_rank, g)
        self.o_b_proj = nn.Linear(g * config.o_lora_rank, config.hidden_size, bias=False)
        self.sinks = nn.Parameter(torch.zeros(self.heads))
        self.compressor = {"sliding_attention": None, "compressed_sparse_attention": CSACompressor,
                           "heavily_compressed_attention": HCACompressor}[self.kind]
        if self.compressor is not None:
            self.compressor = self.compressor(config)

    def forward(self, h: Tensor, layout: PackedLayout) -> Tensor:
        T = h.shape[0]
        cos, sin = layout.rope[self.rope_kind]
        q_res = self.q_a_norm(self.q_a_proj(h))
        q = rms_unweighted(self.q_b_proj(q_res).view(T, self.heads, self.head_dim), self.config.rms_norm_eps)
        q = rope_interleaved(q, cos[:, None], sin[:, None])
        kv = rope_interleaved(self.kv_norm(self.kv_proj(h)), cos, sin)       # [T, d]
        keys, slots = kv, layout.window
        if self.compressor is not None:
            ent, picks = self.compressor(h, q_res, layout)
            keys = torch.cat([kv, ent.to(kv.dtype)], dim=0)
            slots = torch.cat([slots, torch.where(picks >= 0, picks + T, picks)], dim=1)
        o = gathered_attention(q, keys, slots, self.sinks, self.head_dim ** -0.5)
        o = rope_interleaved(o, cos[:, None], -sin[:, None])  # values carried the key rotation
        g = self.config.o_groups
        return self.o_b_proj(self.o_a_proj(o.reshape(T, g, -1)).flatten(1))
