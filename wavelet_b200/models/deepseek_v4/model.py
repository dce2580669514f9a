"""DeepSeek-V4 decoder, eager PyTorch (reference trainer/models/deepseek_v4/
modeling.py).

Forward: token embeddings are copied into ``hc_mult`` residual streams;
every layer runs attention then MoE, each wrapped by a hyper-connection
(collapse -> RMSNorm -> sub-layer -> spread + Sinkhorn remix); a hyper head
collapses the streams, then the final RMSNorm and the LM head.  Batches are
packed into one row: documents are delimited by ``position_ids`` restarting
at 0 (each batch row starts a document), and attention never crosses them.

Checkpoints: ``save_pretrained`` writes config.json (marked
``wavelet_checkpoint_format = deepseek_v4_native_v1``) and
``model.safetensors`` with the native tensor names;
``convert.convert_checkpoint`` maps published (raw) checkpoints to and from
this layout.  Numerically sensitive tensors (hyper-connection maps, sinks,
compressor position biases, routing biases, norms) stay fp32 when the rest
of the model is loaded or transferred in bf16.

Not supported (as in the reference's eager model): context / tensor / expert
parallelism and cached decoding.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .attention import Attention, PackedLayout
from .config import CHECKPOINT_FORMAT, DeepseekV4Config
from .layers import DualRotary, HyperConnection, HyperHead, RMSNorm
from .moe import MoE

FP32_PARTS = ("attn_hc", "ffn_hc", "hc_head", "sinks", "position_bias", "selection_bias", "q_a_norm", "kv_norm",
              "input_layernorm", "post_attention_layernorm", "norm")


@dataclass
class CausalLMOutput:
    loss: Tensor | None
    logits: Tensor


class DecoderLayer(nn.Module):
    def __init__(self, config: DeepseekV4Config, idx: int):
        super().__init__()
        self.self_attn = Attention(config, idx)
        self.mlp = MoE(config, idx)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.attn_hc = HyperConnection(config)
        self.ffn_hc = HyperConnection(config)

    def forward(self, streams: Tensor, ids: Tensor, layout: PackedLayout) -> Tensor:
        """streams [T, hc, H] of one packed row."""
        post, comb, x = self.attn_hc(streams)
        streams = HyperConnection.merge(post, comb, self.self_attn(self.input_layernorm(x), layout), streams)
        post, comb, x = self.ffn_hc(streams)
        return HyperConnection.merge(post, comb, self.mlp(self.post_attention_layernorm(x), ids), streams)


class DeepseekV4Model(nn.Module):
    def __init__(self, config: DeepseekV4Config):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size, config.pad_token_id)
        self.layers = nn.ModuleList(DecoderLayer(config, i) for i in range(config.num_hidden_layers))
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.rotary_emb = DualRotary(config)
        self.hc_head = HyperHead(config)

    def forward(self, ids: Tensor, seq_lens: Tensor) -> Tensor:
        """ids [T] (one packed row), seq_lens [n_docs] -> hidden [T, H]."""
        x = self.embed_tokens(ids)
        layout = PackedLayout.build(self.rotary_emb, seq_lens, x.dtype, x.device)
        streams = x.unsqueeze(1).expand(-1, self.config.hc_mult, -1).contiguous()
        for layer in self.layers:
            streams = layer(streams, ids, layout)
        return self.norm(self.hc_head(streams))


def _doc_lengths(position_ids: Tensor) -> Tensor:
    """Lengths of the documents of a flattened row whose positions restart at 0."""
    flat = position_ids.reshape(-1)
    starts = (flat == 0).nonzero().flatten()
    ends = torch.cat([starts[1:], starts.new_tensor([flat.numel()])])
    return ends - starts


class DeepseekV4ForCausalLM(nn.Module):
    checkpoint_format = CHECKPOINT_FORMAT

    def __init__(self, config: DeepseekV4Config, init: bool = True):
        super().__init__()
        config.set_extra("wavelet_checkpoint_format", self.checkpoint_format)
        self.config = config
        self.model = DeepseekV4Model(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if init:
            self.reset_parameters()

    # ------------------------------------------------------------ weights
    @torch.no_grad()
    def reset_parameters(self) -> None:
        std = self.config.initializer_range
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, std=std)
            elif isinstance(m, (HyperConnection, HyperHead)):
                m.reset_parameters(std)
            elif isinstance(m, RMSNorm):
                nn.init.ones_(m.weight)
        for name, p in self.named_parameters():
            if name.endswith(("experts.gate_proj", "experts.up_proj", "experts.down_proj")):
                nn.init.normal_(p, std=std)
            elif name.endswith(("sinks", "position_bias")):
                nn.init.zeros_(p)

    @classmethod
    def keep_in_fp32_for_weight_transfer(cls, name: str) -> bool:
        return any(part in name for part in FP32_PARTS)

    def to_compute_dtype(self, dtype: torch.dtype) -> "DeepseekV4ForCausalLM":
        """Cast to ``dtype`` except the fp32-sensitive tensors."""
        for name, p in self.named_parameters():
            if not self.keep_in_fp32_for_weight_transfer(name) and p.is_floating_point():
                p.data = p.data.to(dtype)
        for name, b in self.named_buffers():
            if b.is_floating_point() and not self.keep_in_fp32_for_weight_transfer(name) and "inv_freq" not in name:
                b.data = b.data.to(dtype)
        return self

    def save_pretrained(self, path: str | Path) -> None:
        from safetensors.torch import save_file

        p = Path(path)
        p.mkdir(parents=True, exist_ok=True)
        self.config.save_pretrained(p)
        save_file({k: v.detach().contiguous().cpu() for k, v in self.state_dict().items()}, str(p / "model.safetensors"))

    @classmethod
    def from_pretrained(cls, path: str | Path, dtype: torch.dtype | None = None, device="cpu") -> "DeepseekV4ForCausalLM":
        from safetensors.torch import load_file

        p = Path(path)
        cfg = DeepseekV4Config.from_pretrained(p)
        if getattr(cfg, "wavelet_checkpoint_format", None) != CHECKPOINT_FORMAT:
            raise ValueError(f"{p} is not a converted native checkpoint (convert published weights with "
                             "wavelet_b200.models.deepseek_v4.convert first)")
        model = cls(cfg, init=False)
        model.load_state_dict(load_file(str(p / "model.safetensors"), device=str(device)), strict=True)
        model.to(device)
        if dtype is not None:
            model.to_compute_dtype(dtype)
        return model

    def load_state_dict(self, state, strict: bool = True, assign: bool = False):
        out = super().load_state_dict(state, strict=strict, assign=assign)
        for m in self.modules():
            if isinstance(m, DualRotary):
                m.reset_tables()
            if isinstance(m, MoE):
                m.tokens_per_expert.zero_()
        return out

    # ------------------------------------------------------------ forward
    def hidden(self, input_ids: Tensor, position_ids: Tensor | None = None) -> Tensor:
        B, L = input_ids.shape
        if L == 0:
            raise ValueError("DeepSeek-V4 needs a non-empty sequence")
        if position_ids is None:
            position_ids = torch.arange(L, device=input_ids.device).expand(B, -1)
        if position_ids.shape != input_ids.shape or bool((position_ids[:, 0] != 0).any()):
            raise ValueError("DeepSeek-V4 positions must match the inputs and start at 0 in every row")
        lens = _doc_lengths(position_ids)
        expect = torch.cat([torch.arange(int(n), device=input_ids.device) for n in lens.tolist()])
        if not torch.equal(expect, position_ids.reshape(-1).to(expect.dtype)):
            raise ValueError("DeepSeek-V4 positions must count up by one inside every document")
        return self.model(input_ids.reshape(-1), lens).view(B, L, -1)

    def forward(self, input_ids: Tensor, attention_mask: Tensor | None = None, position_ids: Tensor | None = None,
                labels: Tensor | None = None, use_cache: bool = False, **kwargs) -> CausalLMOutput:
        if use_cache or kwargs.get("past_key_values") is not None:
            raise ValueError("the eager DeepSeek-V4 model has no cached decoding")
        if attention_mask is not None:
            if attention_mask.shape != input_ids.shape:
                raise ValueError("DeepSeek-V4 accepts a 2-D right-padding mask only")
            if bool((attention_mask[:, 1:].int() > attention_mask[:, :-1].int()).any()):
                raise ValueError("DeepSeek-V4 eager training requires right padding")
        logits = self.lm_head(self.hidden(input_ids, position_ids))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[:, :-1].float().reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1))
        return CausalLMOutput(loss, logits)

    @torch.no_grad()
    def balance_experts_(self, rate: float = 1e-3) -> None:
        """Apply the auxiliary-loss-free routing-bias update of every top-k
        MoE layer (call once per optimizer step)."""
        for m in self.modules():
            if isinstance(m, MoE):
                m.balance_(rate)
