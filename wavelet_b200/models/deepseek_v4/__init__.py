"""Eager DeepSeek-V4 (sliding / compressed-sparse / heavily-compressed
attention, hyper-connections, hash and top-k routed MoE) with native
checkpoints and conversion from the published layout."""

from .config import DeepseekV4Config
from .model import DeepseekV4ForCausalLM

__all__ = ["DeepseekV4Config", "DeepseekV4ForCausalLM"]
