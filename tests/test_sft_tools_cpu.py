"""Tool schemas and chat-template arguments of SFT / RL rows
(data.tools_column, data.chat_template_kwargs_column; ref data/sft.py:259-310,
393-440): they reach every chat-template call, and tool-call arguments stored
as JSON text are decoded before rendering."""

from __future__ import annotations

import json
import pytest


class _TemplateTok:
    """Renders messages as text; the tool names and enable_thinking show in the output."""

    def __init__(self):
        self.calls = []

    def apply_chat_template(self, msgs, tokenize=True, add_generation_prompt=False, tools=None, **kw):
        self.calls.append({"tools": tools, **kw})
        head = "T:" + ",".join(t["function"]["name"] for t in tools) + "|" if tools else ""
        head += "nothink|" if kw.get("enable_thinking") is False else ""
        body = "".join(f"<{m['role']}>{m.get('content') or ''}{json.dumps(m.get('tool_calls')) if m.get('tool_calls') else ''}"
                       for m in msgs)
        text = head + body + ("<assistant>" if add_generation_prompt else "")
        return [ord(c) for c in text]


def _cfg(**kw):
    from wavelet_b200.configs.config import SFTConfig

    return SFTConfig.model_validate({"data": {"source": "local", **kw}}).data


TOOLS = [{"type": "function", "function": {"name": "lookup", "parameters": {"type": "object"}}}]


def test_rows_pass_tools_and_template_arguments():
    from wavelet_b200.data.sft import normalize_messages, template_kwargs, tokenize_messages

    cfg = _cfg(tools_column="my_tools")
    row = {"messages": [{"role": "user", "content": "hi"},
                        {"role": "assistant", "content": "", "tool_calls": [
                            {"type": "function", "function": {"name": "lookup", "arguments": "{\"q\": 1}"}}]}],
           "my_tools": TOOLS, "chat_template_kwargs": {"enable_thinking": False}}
    kw = template_kwargs(row, cfg)
    assert kw == {"tools": TOOLS, "enable_thinking": False}
    msgs = normalize_messages(row, cfg)
    assert msgs[1]["tool_calls"][0]["function"]["arguments"] == {"q": 1}  # JSON text decoded
    tok = _TemplateTok()
    s = tokenize_messages(msgs, tok, cfg, kw)
    text = "".join(chr(i) for i in s.input_ids)
    assert text.startswith("T:lookup|nothink|<user>hi")
    assert all(c["tools"] == TOOLS and c["enable_thinking"] is False for c in tok.calls)
    # the assistant turn (with its tool call) is trained, the prompt is not
    trained = "".join(chr(i) for i, m in zip(s.input_ids, s.loss_mask) if m)
    assert "lookup" in trained and "hi" not in trained


def test_bad_tool_and_kwargs_columns_are_refused():
    from wavelet_b200.data.sft import template_kwargs

    cfg = _cfg()
    with pytest.raises(ValueError, match="tools must be a list"):
        template_kwargs({"tools": {"a": 1}}, cfg)
    with pytest.raises(ValueError, match="chat_template_kwargs must be an object"):
        template_kwargs({"chat_template_kwargs": [1]}, cfg)
    assert template_kwargs({"tools": json.dumps(TOOLS)}, cfg) == {"tools": TOOLS}


def test_rl_prompt_rows_and_records_render_tools(tmp_path):
    from wavelet_b200.data.rl import RLExample, example_from_payload, example_to_payload
    from wavelet_b200.inference.policy import record_prompt_ids
    from wavelet_b200.orchestrator.sources import FilePromptSource

    rows = tmp_path / "p.jsonl"
    rows.write_text(json.dumps({"prompt": [{"role": "user", "content": "q"}], "tools": TOOLS,
                                "chat_template_kwargs": {"enable_thinking": False}}) + "\n")
    from wavelet_b200.configs.config import RLConfig

    cfg = RLConfig.model_validate({"data": {"source": "local", "path": str(rows)}})
    tok = _TemplateTok()
    src = FilePromptSource(cfg, tokenizer=tok)
    rec = src.take(1)[0]
    assert "".join(chr(i) for i in rec.prompt_ids).startswith("T:lookup|nothink|<user>q")
    # a rollout record carries its tools through the queue and into prompt rendering
    ex = RLExample(prompt=[{"role": "user", "content": "q"}], completion=[], advantage=None, reward=None,
                   tools=TOOLS, chat_template_kwargs={"enable_thinking": False})
    row = example_to_payload(ex, cfg.data.model_copy(update={"tools_column": "tool_schemas"}))
    assert "tool_schemas" in row and "tools" not in row
    back = example_from_payload(row, cfg.data.model_copy(update={"tools_column": "tool_schemas"}))
    assert back.tools == TOOLS
    ids = record_prompt_ids(back, tok)
    assert "".join(chr(i) for i in ids).startswith("T:lookup|nothink|")
