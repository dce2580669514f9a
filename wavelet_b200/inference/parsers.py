"""Chat-output parsers of the OpenAI server: reasoning and tool calls.

The reference hands ``inference.vllm.reasoning_parser`` and
``tool_call_parser`` to ``vllm serve`` (inference/server.py:1162-1174), whose
parsers split a completion into ``reasoning_content``, ``content`` and
``tool_calls``.  The native server has no vLLM, so the formats those names
stand for are parsed here, on the decoded completion text:

reasoning parsers (``<think>`` ... ``</think>``):
    ``deepseek_r1`` / ``nemotron_v3`` / ``minimax_m2``: everything before
    ``</think>`` is reasoning; a completion cut off before ``</think>`` is all
    reasoning (the prompt opened the think block).  ``nemotron_v3`` with
    ``enable_thinking: false`` in the chat-template arguments has no reasoning.
    ``qwen3`` / ``glm45``: reasoning only when the block is closed; otherwise
    the text is content.  ``minimax_m2_append_think``: no split, the content
    gets the ``<think>`` the prompt ended with put back in front.
tool-call parsers:
    ``hermes``       ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>``
    ``qwen3_coder``  ``<tool_call><function=NAME><parameter=KEY>VALUE</parameter>
                     </function></tool_call>``
    ``glm45``/``glm47`` ``<tool_call>NAME<arg_key>KEY</arg_key><arg_value>VALUE
                     </arg_value></tool_call>``
    ``minimax_m2``   ``<minimax:tool_call><invoke name="NAME"><parameter
                     name="KEY">VALUE</parameter></invoke></minimax:tool_call>``

Parameter values of the XML-style formats are converted with the request's
tool schema (``string`` stays text; ``integer``, ``number``, ``boolean``,
``object``, ``array`` and ``null`` are parsed).  A completion whose calls do
not parse is returned as plain content, as vLLM does.

``"auto"`` resolves the parser from the model name by family
(ref ``MODEL_TOOL_CALL_PARSER`` / ``MODEL_REASONING_PARSER_PATTERNS``,
inference/server.py:64-159): Qwen3 and INTELLECT-3 use ``hermes``, the Qwen3.5
family and Nemotron-3 use ``qwen3_coder``, GLM-4.5 ``glm45``, GLM-4.7 / GLM-5
``glm47``, MiniMax-M2 ``minimax_m2``; other names get no parser.
"""

from __future__ import annotations

import ast
import json
import re
import uuid
from dataclasses import dataclass, field
from typing import Any, Callable

THINK_START = "<think>"
THINK_END = "</think>"

# family rules: (pattern on the model name, parser)
_TOOL_RULES: tuple[tuple[re.Pattern[str], str], ...] = (
    (re.compile(r"^zai-org/GLM-4\.5"), "glm45"),
    (re.compile(r"^zai-org/GLM-(4\.7|5)"), "glm47"),
    (re.compile(r"^MiniMaxAI/MiniMax-M2"), "minimax_m2"),
    (re.compile(r"^PrimeIntellect/INTELLECT-3"), "hermes"),
    (re.compile(r"^Qwen/Qwen3\.5-"), "qwen3_coder"),
    (re.compile(r"^nvidia/NVIDIA-Nemotron-3-"), "qwen3_coder"),
    (re.compile(r"^Qwen/Qwen3-"), "hermes"),
)
_REASONING_RULES: tuple[tuple[re.Pattern[str], str], ...] = (
    (re.compile(r"^zai-org/GLM-"), "glm45"),
    (re.compile(r"^MiniMaxAI/MiniMax-M2"), "minimax_m2_append_think"),
    (re.compile(r"^PrimeIntellect/INTELLECT-3"), "deepseek_r1"),
    (re.compile(r"^nvidia/NVIDIA-Nemotron-3-Super"), "nemotron_v3"),
    (re.compile(r"^Qwen/Qwen3-.*Thinking"), "deepseek_r1"),
    (re.compile(r"^Qwen/Qwen3\.(5|6|8)-"), "qwen3"),
)


def resolve_tool_call_parser(model_name: str, setting: str | None) -> str | None:
    """The tool-call parser for ``setting`` (``"auto"`` resolves by model family)."""
    if setting != "auto":
        return setting
    for pat, name in _TOOL_RULES:
        if pat.search(model_name):
            return name
    return None


def resolve_reasoning_parser(model_name: str, setting: str | None) -> str | None:
    """The reasoning parser for ``setting`` (``"auto"`` resolves by model family)."""
    if setting != "auto":
        return setting
    for pat, name in _REASONING_RULES:
        if pat.search(model_name):
            return name
    return None


# ----------------------------------------------------------------------------------------------------------------
# reasoning
# ----------------------------------------------------------------------------------------------------------------


def _strip_open(text: str) -> str:
    s = text.lstrip()
    return s[len(THINK_START):] if s.startswith(THINK_START) else text


def _split_closed(text: str) -> tuple[str | None, str | None] | None:
    """(reasoning, content) when the think block is closed, else None."""
    body = _strip_open(text)
    if THINK_END not in body:
        return None
    reasoning, _, content = body.partition(THINK_END)
    return reasoning, (content.lstrip("\n") or None)


def _reason_open_ended(text: str, kwargs: dict[str, Any]) -> tuple[str | None, str | None]:
    split = _split_closed(text)
    if split is not None:
        return split
    return _strip_open(text), None


def _reason_closed_only(text: str, kwargs: dict[str, Any]) -> tuple[str | None, str | None]:
    split = _split_closed(text)
    if split is not None:
        return split
    return None, text


def _reason_nemotron(text: str, kwargs: dict[str, Any]) -> tuple[str | None, str | None]:
    if kwargs.get("enable_thinking") is False:
        return None, text
    return _reason_open_ended(text, kwargs)


def _reason_append_think(text: str, kwargs: dict[str, Any]) -> tuple[str | None, str | None]:
    return None, (text if text.lstrip().startswith(THINK_START) else THINK_START + text)


REASONING_PARSERS: dict[str, Callable[[str, dict[str, Any]], tuple[str | None, str | None]]] = {
    "deepseek_r1": _reason_open_ended,
    "minimax_m2": _reason_open_ended,
    "nemotron_v3": _reason_nemotron,
    "qwen3": _reason_closed_only,
    "glm45": _reason_closed_only,
    "minimax_m2_append_think": _reason_append_think,
}


# ----------------------------------------------------------------------------------------------------------------
# tool calls
# ----------------------------------------------------------------------------------------------------------------


def _param_types(tools: list[dict[str, Any]] | None, name: str) -> dict[str, Any]:
    for t in tools or []:
        fn = t.get("function", t) if isinstance(t, dict) else {}
        if fn.get("name") == name:
            props = (fn.get("parameters") or {}).get("properties") or {}
            return {k: (v or {}).get("type") for k, v in props.items() if isinstance(v, dict)}
    return {}


def _convert(value: str, typ: Any) -> Any:
    """A parameter's text as the JSON type its schema names (text if none parses)."""
    if isinstance(typ, list):  # ["integer", "null"] and the like
        for t in typ:
            if t == "null" and value.strip().lower() in ("null", "none"):
                return None
        typ = next((t for t in typ if t != "null"), "string")
    if typ in (None, "string"):
        return value
    v = value.strip()
    if v.lower() in ("null", "none") and typ != "string":
        return None
    try:
        if typ == "integer":
            return int(v)
        if typ == "number":
            f = float(v)
            return int(f) if f.is_integer() and "." not in v and "e" not in v.lower() else f
        if typ == "boolean":
            if v.lower() in ("true", "false"):
                return v.lower() == "true"
            raise ValueError(v)
        return json.loads(v)
    except (ValueError, json.JSONDecodeError):
        try:
            return ast.literal_eval(v)
        except (ValueError, SyntaxError):
            return value


def _strip_one_newline(s: str) -> str:
    if s.startswith("\n"):
        s = s[1:]
    if s.endswith("\n"):
        s = s[:-1]
    return s


@dataclass
class ToolCall:
    name: str
    arguments: dict[str, Any]
    id: str = field(default_factory=lambda: "call_" + uuid.uuid4().hex[:24])

    def to_openai(self) -> dict[str, Any]:
        return {"id": self.id, "type": "function",
                "function": {"name": self.name, "arguments": json.dumps(self.arguments, ensure_ascii=False)}}


def _blocks(text: str, start: str, end: str) -> tuple[str, list[str]] | None:
    """Content before the first ``start`` and the body of every block (the last
    one may be unterminated), or None when ``start`` does not occur."""
    i = text.find(start)
    if i < 0:
        return None
    bodies = []
    pos = i
    while pos >= 0:
        s = pos + len(start)
        e = text.find(end, s)
        if e < 0:
            bodies.append(text[s:])
            break
        bodies.append(text[s:e])
        pos = text.find(start, e + len(end))
    return text[:i], bodies


def _tools_hermes(text: str, tools) -> tuple[str, list[ToolCall]] | None:
    found = _blocks(text, "<tool_call>", "</tool_call>")
    if found is None:
        return None
    content, bodies = found
    calls = []
    for b in bodies:
        obj = json.loads(b.strip())
        args = obj.get("arguments", obj.get("parameters", {}))
        if isinstance(args, str):
            args = json.loads(args)
        calls.append(ToolCall(str(obj["name"]), dict(args)))
    return content, calls


_QC_FN = re.compile(r"<function=([^>\n]+)>(.*?)(?:</function>|$)", re.S)
_QC_PARAM = re.compile(r"<parameter=([^>\n]+)>(.*?)(?:</parameter>|(?=<parameter=)|(?=</function>)|$)", re.S)


def _tools_qwen3_coder(text: str, tools) -> tuple[str, list[ToolCall]] | None:
    found = _blocks(text, "<tool_call>", "</tool_call>")
    if found is None:
        return None
    content, bodies = found
    calls = []
    for b in bodies:
        m = _QC_FN.search(b)
        if m is None:
            raise ValueError("tool call without <function=...>")
        name = m.group(1).strip()
        types = _param_types(tools, name)
        args = {k.strip(): _convert(_strip_one_newline(v), types.get(k.strip()))
                for k, v in _QC_PARAM.findall(m.group(2))}
        calls.append(ToolCall(name, args))
    return content, calls


_GLM_ARG = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)(?:</arg_value>|$)", re.S)


def _tools_glm(text: str, tools) -> tuple[str, list[ToolCall]] | None:
    found = _blocks(text, "<tool_call>", "</tool_call>")
    if found is None:
        return None
    content, bodies = found
    calls = []
    for b in bodies:
        k = b.find("<arg_key>")
        name = (b if k < 0 else b[:k]).strip()
        if not name:
            raise ValueError("tool call without a function name")
        types = _param_types(tools, name)
        args = {}
        for key, val in _GLM_ARG.findall(b):
            key = key.strip()
            typ = types.get(key)
            args[key] = _convert(val, typ if typ is not None else "json-or-text")
        calls.append(ToolCall(name, args))
    return content, calls


_MM_INVOKE = re.compile(r"<invoke\s+name=\"?([^\">]+)\"?\s*>(.*?)(?:</invoke>|$)", re.S)
_MM_PARAM = re.compile(r"<parameter\s+name=\"?([^\">]+)\"?\s*>(.*?)(?:</parameter>|$)", re.S)


def _tools_minimax(text: str, tools) -> tuple[str, list[ToolCall]] | None:
    found = _blocks(text, "<minimax:tool_call>", "</minimax:tool_call>")
    if found is None:
        return None
    content, bodies = found
    calls = []
    for b in bodies:
        for name, inner in _MM_INVOKE.findall(b):
            name = name.strip()
            types = _param_types(tools, name)
            args = {k.strip(): _convert(v.strip("\n"), types.get(k.strip())) for k, v in _MM_PARAM.findall(inner)}
            calls.append(ToolCall(name, args))
    if not calls:
        raise ValueError("tool-call block without an <invoke>")
    return content, calls


TOOL_PARSERS: dict[str, Callable[[str, Any], tuple[str, list[ToolCall]] | None]] = {
    "hermes": _tools_hermes,
    "qwen3_coder": _tools_qwen3_coder,
    "glm45": _tools_glm,
    "glm47": _tools_glm,
    "minimax_m2": _tools_minimax,
}


def _check(name: str | None, table: dict[str, Any], what: str) -> None:
    if name is not None and name not in table:
        raise ValueError(f"unknown {what} {name!r}; the native server parses {sorted(table)}")


@dataclass
class ParsedChat:
    content: str | None
    reasoning_content: str | None
    tool_calls: list[ToolCall]

    def message(self) -> dict[str, Any]:
        msg: dict[str, Any] = {"role": "assistant", "content": self.content}
        if self.reasoning_content is not None:
            msg["reasoning_content"] = self.reasoning_content
        if self.tool_calls:
            msg["tool_calls"] = [c.to_openai() for c in self.tool_calls]
        return msg


class ChatOutputParser:
    """Splits a decoded chat completion into reasoning, content and tool calls."""

    def __init__(self, reasoning_parser: str | None, tool_call_parser: str | None):
        _check(reasoning_parser, REASONING_PARSERS, "reasoning parser")
        _check(tool_call_parser, TOOL_PARSERS, "tool-call parser")
        self.reasoning_parser = reasoning_parser
        self.tool_call_parser = tool_call_parser

    @classmethod
    def for_model(cls, model_name: str, reasoning_setting: str | None, tool_setting: str | None) -> "ChatOutputParser":
        return cls(resolve_reasoning_parser(model_name, reasoning_setting),
                   resolve_tool_call_parser(model_name, tool_setting))

    def parse(self, text: str, *, tools: list[dict[str, Any]] | None = None, tool_choice: Any = "auto",
              include_reasoning: bool = True, chat_template_kwargs: dict[str, Any] | None = None) -> ParsedChat:
        reasoning, content = None, text
        if self.reasoning_parser is not None:
            reasoning, content = REASONING_PARSERS[self.reasoning_parser](text, chat_template_kwargs or {})
        if not include_reasoning:
            reasoning = None
        calls: list[ToolCall] = []
        if self.tool_call_parser is not None and content and tools and tool_choice != "none":
            try:
                got = TOOL_PARSERS[self.tool_call_parser](content, tools)
            except (ValueError, KeyError, TypeError, json.JSONDecodeError):
                got = None  # malformed calls stay content
            if got is not None and got[1]:
                pre, calls = got
                content = pre.strip() or None
        return ParsedChat(content if content else None, reasoning, calls)
