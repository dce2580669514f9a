"""Tokenizers.

* ``CharTokenizer`` — a dependency-free byte/character tokenizer with a tiny
  chat template, used by the debug model and CPU tests (the reference's debug
  character tokenizer, trainer/debug.py:26-115).
* ``load_tokenizer`` — a Hugging Face tokenizer from a local directory
  (``transformers.AutoTokenizer``, no network), or the char tokenizer for
  presets / the debug model.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any


class CharTokenizer:
    """UTF-8 byte tokenizer: ids 0..2 are <pad>, <bos>, <eos>; bytes map to 3..258."""

    pad_token_id = 0
    bos_token_id = 1
    eos_token_id = 2
    vocab_size = 259
    ROLE_TAGS = {"system": "<|system|>", "user": "<|user|>", "assistant": "<|assistant|>", "tool": "<|tool|>"}

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids = [b + 3 for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids: list[int], skip_special_tokens: bool = True) -> str:
        out = bytes(i - 3 for i in ids if 3 <= i < 259)
        return out.decode("utf-8", errors="replace")

    def __call__(self, text: str, add_special_tokens: bool = False, **_: Any) -> dict[str, list[int]]:
        return {"input_ids": self.encode(text, add_special_tokens)}

    def role_header(self, role: str) -> str:
        return self.ROLE_TAGS.get(role, "<|" + role + "|>")

    def render_message(self, role: str, content: str) -> str:
        return f"{self.role_header(role)}{content}\n"

    def apply_chat_template(self, messages: list[dict[str, Any]], tokenize: bool = False,
                            add_generation_prompt: bool = False, **_: Any):
        text = "".join(self.render_message(m["role"], str(m.get("content") or "")) for m in messages)
        if add_generation_prompt:
            text += self.ROLE_TAGS["assistant"]
        return self.encode(text) if tokenize else text


def load_tokenizer(name_or_path: str | Path, trust_remote_code: bool = False, chat_template: str | None = None):
    """The tokenizer of a local model directory (or the char tokenizer of the
    synthetic presets).  ``chat_template``: a Jinja template, or the path of a
    file holding one, that replaces the directory's template."""
    p = Path(str(name_or_path))
    if p.is_dir() and ((p / "tokenizer.json").exists() or (p / "tokenizer_config.json").exists()):
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(str(p), trust_remote_code=trust_remote_code, local_files_only=True)
        if tok.pad_token_id is None:
            tok.pad_token = tok.eos_token
        if chat_template:
            t = Path(chat_template)
            tok.chat_template = t.read_text() if t.is_file() else chat_template
        return tok
    if chat_template:
        raise ValueError(f"model.chat_template needs a Hugging Face tokenizer; {name_or_path} has none")
    return CharTokenizer()


def tokenizer_for(model_cfg):
    """``load_tokenizer`` with the model section's template and remote-code settings."""
    return load_tokenizer(model_cfg.name, trust_remote_code=bool(getattr(model_cfg, "trust_remote_code", False)),
                          chat_template=getattr(model_cfg, "chat_template", None))
