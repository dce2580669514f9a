"""Reasoning and tool-call parsers of the native OpenAI server.

The formats are the ones the reference's parser names select in vLLM
(ref inference/server.py:64-174): each case is a completion text as the model
family writes it and the message the server must return.
"""

from __future__ import annotations

import json
from dataclasses import dataclass

import pytest

from wavelet_b200.inference.parsers import (ChatOutputParser, resolve_reasoning_parser,
                                            resolve_tool_call_parser)

WEATHER = [{"type": "function", "function": {
    "name": "get_weather",
    "parameters": {"type": "object", "properties": {
        "city": {"type": "string"}, "days": {"type": "integer"}, "metric": {"type": "boolean"},
        "hours": {"type": "array"}, "scale": {"type": "number"}, "note": {"type": ["string", "null"]}}}}}]


def _args(msg, i=0):
    return json.loads(msg["tool_calls"][i]["function"]["arguments"])


@pytest.mark.parametrize("name,tool,reason", [
    ("Qwen/Qwen3-4B", "hermes", None),
    ("Qwen/Qwen3-30B-A3B-Thinking-2507", "hermes", "deepseek_r1"),
    ("Qwen/Qwen3.5-9B", "qwen3_coder", "qwen3"),
    ("nvidia/NVIDIA-Nemotron-3-Super-120B-A12B-BF16", "qwen3_coder", "nemotron_v3"),
    ("zai-org/GLM-4.5-Air", "glm45", "glm45"),
    ("zai-org/GLM-4.7", "glm47", "glm45"),
    ("zai-org/GLM-5.1-FP8", "glm47", "glm45"),
    ("MiniMaxAI/MiniMax-M2.1", "minimax_m2", "minimax_m2_append_think"),
    ("PrimeIntellect/INTELLECT-3", "hermes", "deepseek_r1"),
    ("meta-llama/Llama-3.1-8B", None, None),
    ("/local/dir/model", None, None),
])
def test_auto_resolution(name, tool, reason):
    assert resolve_tool_call_parser(name, "auto") == tool
    assert resolve_reasoning_parser(name, "auto") == reason
    assert resolve_tool_call_parser(name, "hermes") == "hermes"
    assert resolve_reasoning_parser(name, None) is None


def test_unknown_parser_is_refused():
    with pytest.raises(ValueError, match="unknown tool-call parser"):
        ChatOutputParser(None, "nope")
    with pytest.raises(ValueError, match="unknown reasoning parser"):
        ChatOutputParser("nope", None)


def test_reasoning_variants():
    r1 = ChatOutputParser("deepseek_r1", None)
    m = r1.parse("<think>plan it</think>\n\nanswer 4").message()
    assert m["reasoning_content"] == "plan it" and m["content"] == "answer 4"
    m = r1.parse("still thinking when cut off").message()  # the prompt opened the block
    assert m["reasoning_content"] == "still thinking when cut off" and m["content"] is None
    q3 = ChatOutputParser("qwen3", None)
    m = q3.parse("no think block here").message()
    assert m["content"] == "no think block here" and "reasoning_content" not in m
    m = q3.parse("<think>\nx\n</think>\n\ny").message()
    assert m["reasoning_content"] == "\nx\n" and m["content"] == "y"
    nem = ChatOutputParser("nemotron_v3", None)
    assert nem.parse("a</think>b").message()["reasoning_content"] == "a"
    m = nem.parse("a</think>b", chat_template_kwargs={"enable_thinking": False}).message()
    assert m["content"] == "a</think>b" and "reasoning_content" not in m
    mm = ChatOutputParser("minimax_m2_append_think", None)
    assert mm.parse("r</think>c").message()["content"] == "<think>r</think>c"
    # include_reasoning: false drops the reasoning, keeps the content
    m = r1.parse("<think>a</think>b", include_reasoning=False).message()
    assert m["content"] == "b" and "reasoning_content" not in m


def test_hermes_tool_calls():
    p = ChatOutputParser(None, "hermes")
    text = ('Let me check.\n<tool_call>\n{"name": "get_weather", "arguments": {"city": "Paris", "days": 2}}\n'
            '</tool_call>\n<tool_call>\n{"name": "get_weather", "arguments": {"city": "Oslo"}}\n</tool_call>')
    m = p.parse(text, tools=WEATHER).message()
    assert m["content"] == "Let me check."
    assert [c["function"]["name"] for c in m["tool_calls"]] == ["get_weather", "get_weather"]
    assert _args(m, 0) == {"city": "Paris", "days": 2} and _args(m, 1) == {"city": "Oslo"}
    assert m["tool_calls"][0]["id"] != m["tool_calls"][1]["id"] and m["tool_calls"][0]["type"] == "function"
    # no tools in the request / tool_choice none / malformed JSON: plain content
    assert "tool_calls" not in p.parse(text).message()
    assert "tool_calls" not in p.parse(text, tools=WEATHER, tool_choice="none").message()
    bad = "<tool_call>{not json}</tool_call>"
    assert p.parse(bad, tools=WEATHER).message() == {"role": "assistant", "content": bad}
    # an unterminated last call (cut at max_tokens) still parses when its JSON is whole
    m = p.parse('<tool_call>{"name": "get_weather", "arguments": {"city": "Rome"}}', tools=WEATHER).message()
    assert _args(m) == {"city": "Rome"} and m["content"] is None


def test_qwen3_coder_tool_calls_convert_by_schema():
    p = ChatOutputParser(None, "qwen3_coder")
    text = ("Sure.\n<tool_call>\n<function=get_weather>\n<parameter=city>\nNew York\n</parameter>\n"
            "<parameter=days>\n3\n</parameter>\n<parameter=metric>\ntrue\n</parameter>\n"
            "<parameter=hours>\n[1, 2]\n</parameter>\n<parameter=scale>\n1.5\n</parameter>\n"
            "<parameter=note>\nnull\n</parameter>\n<parameter=extra>\n42\n</parameter>\n"
            "</function>\n</tool_call>")
    m = p.parse(text, tools=WEATHER).message()
    assert m["content"] == "Sure."
    assert _args(m) == {"city": "New York", "days": 3, "metric": True, "hours": [1, 2], "scale": 1.5,
                        "note": None, "extra": "42"}


def test_glm_tool_calls():
    for name in ("glm45", "glm47"):
        p = ChatOutputParser("glm45", name)
        sep = "\n" if name == "glm45" else ""
        text = (f"<think>need weather</think>\nok<tool_call>get_weather{sep}<arg_key>city</arg_key>{sep}"
                f"<arg_value>Lima</arg_value>{sep}<arg_key>days</arg_key>{sep}<arg_value>5</arg_value>{sep}"
                f"<arg_key>hours</arg_key>{sep}<arg_value>[3]</arg_value>{sep}</tool_call>")
        m = p.parse(text, tools=WEATHER).message()
        assert m["reasoning_content"] == "need weather" and m["content"] == "ok"
        assert m["tool_calls"][0]["function"]["name"] == "get_weather"
        assert _args(m) == {"city": "Lima", "days": 5, "hours": [3]}


def test_minimax_tool_calls():
    p = ChatOutputParser(None, "minimax_m2")
    text = ('pre\n<minimax:tool_call>\n<invoke name="get_weather">\n<parameter name="city">Cairo</parameter>\n'
            '<parameter name="metric">false</parameter>\n</invoke>\n<invoke name="get_weather">\n'
            '<parameter name="city">Doha</parameter>\n</invoke>\n</minimax:tool_call>')
    m = p.parse(text, tools=WEATHER).message()
    assert m["content"] == "pre"
    assert _args(m, 0) == {"city": "Cairo", "metric": False} and _args(m, 1) == {"city": "Doha"}


@dataclass
class _Comp:
    token_ids: list[int]
    logprobs: list[float]
    finish_reason: str = "stop"
    prompt_index: int = 0


class _StubGen:
    max_model_len = 64

    def kv_usage(self):
        return 0.0


class _StubEngine:
    """Returns a fixed completion text so the route's parsing is checked."""
    policy_step = 0

    def __init__(self, tok, text):
        self.generator = _StubGen()
        self.text = text
        self.tok = tok
        self.calls = []

    def generate_ids(self, prompts, ov):
        self.calls.append((prompts, ov))
        ids = self.tok.encode(self.text)
        return [_Comp(ids, [-0.5] * len(ids))]


def test_chat_route_parses_and_fits_context(tmp_path):
    from fastapi.testclient import TestClient

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.data.tokenizer import CharTokenizer
    from wavelet_b200.inference.server import build_app

    cfg = RLConfig.model_validate({
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64, "fake_prompt_len": 6},
        "inference": {"sampling": {"max_completion_tokens": 500},
                      "vllm": {"server_backend": "offline", "reasoning_parser": "deepseek_r1",
                               "tool_call_parser": "hermes"}},
        "lora": None, "output_dir": str(tmp_path / "out")})
    tok = CharTokenizer()
    text = '<think>why</think>call:<tool_call>{"name": "get_weather", "arguments": {"city": "Bern"}}</tool_call>'
    eng = _StubEngine(tok, text)
    c = TestClient(build_app(cfg, engine=eng))
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "tools": WEATHER})
    assert r.status_code == 200
    ch = r.json()["choices"][0]
    assert ch["finish_reason"] == "tool_calls" and ch["message"]["reasoning_content"] == "why"
    assert ch["message"]["content"] == "call:" and _args(ch["message"]) == {"city": "Bern"}
    prompt = r.json()["prompt_token_ids"]
    # max_tokens fitted: 64-token context, the prompt, 16 tokens kept free
    assert eng.calls[-1][1]["max_tokens"] == 64 - len(prompt) - 16
    # the tokens routes take the rendered prompt as is
    r = c.post("/v1/chat/completions/tokens", json={"messages": [], "tokens": [5, 6, 7], "max_tokens": 4})
    assert r.json()["prompt_token_ids"] == [5, 6, 7] and eng.calls[-1][0] == [[5, 6, 7]]
    assert eng.calls[-1][1]["max_tokens"] == 4 and r.json()["usage"]["prompt_tokens"] == 3
    # a prompt that fills the context is refused with the context-length message
    r = c.post("/chat/completions/tokens", json={"messages": [], "tokens": list(range(3, 67))})
    assert r.status_code == 400 and "maximum context length is 64" in r.json()["detail"]


def test_streamed_chat_and_completion_responses(tmp_path):
    import json as _json

    from fastapi.testclient import TestClient

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.data.tokenizer import CharTokenizer
    from wavelet_b200.inference.server import build_app

    cfg = RLConfig.model_validate({
        "model": {"name": "tiny", "random_init": True},
        "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64, "fake_prompt_len": 6},
        "inference": {"vllm": {"server_backend": "offline", "reasoning_parser": "deepseek_r1",
                               "tool_call_parser": "hermes"}},
        "lora": None, "output_dir": str(tmp_path / "out")})
    tok = CharTokenizer()
    eng = _StubEngine(tok, '<think>r</think>hi<tool_call>{"name": "get_weather", "arguments": {}}</tool_call>')
    c = TestClient(build_app(cfg, engine=eng))
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "tools": WEATHER,
                                             "stream": True})
    assert r.headers["content-type"].startswith("text/event-stream")
    events = [line[6:] for line in r.text.splitlines() if line.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [_json.loads(e) for e in events[:-1]]
    deltas = [ch["choices"][0]["delta"] for ch in chunks if ch["choices"]]
    assert deltas[0] == {"role": "assistant"} and {"reasoning_content": "r"} in deltas
    assert {"content": "hi"} in [{k: v for k, v in d.items() if k == "content"} for d in deltas if "content" in d]
    assert any("tool_calls" in d and d["tool_calls"][0]["function"]["name"] == "get_weather" for d in deltas)
    assert [ch["choices"][0]["finish_reason"] for ch in chunks if ch["choices"]][-1] == "tool_calls"
    assert chunks[-1]["usage"]["completion_tokens"] > 0 and all(ch["object"] == "chat.completion.chunk" for ch in chunks)
    r = c.post("/v1/completions", json={"prompt_token_ids": [1, 2], "stream": True})
    events = [line[6:] for line in r.text.splitlines() if line.startswith("data: ")]
    assert events[-1] == "[DONE]" and _json.loads(events[0])["choices"][0]["token_ids"]


def test_stop_strings_cut_the_completion():
    from wavelet_b200.data.tokenizer import CharTokenizer
    from wavelet_b200.inference.server import apply_stop_strings

    tok = CharTokenizer()
    ids = tok.encode("answer: 42\nEND and more")
    lps = [-0.1 * i for i in range(len(ids))]
    out_ids, out_lps, text, hit = apply_stop_strings(tok, ids, lps, ["\nEND", "zzz"])
    assert hit and text == "answer: 42" and tok.decode(out_ids) == "answer: 42\nEND"
    assert out_lps == lps[: len(out_ids)]
    assert apply_stop_strings(tok, ids, lps, "nothing")[3] is False
    # the earliest of several stop strings wins
    assert apply_stop_strings(tok, ids, lps, ["more", ":"])[2] == "answer"


def test_chat_route_applies_stop_strings(tmp_path):
    from fastapi.testclient import TestClient

    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.data.tokenizer import CharTokenizer
    from wavelet_b200.inference.server import build_app

    cfg = RLConfig.model_validate({"model": {"name": "tiny", "random_init": True},
                                   "data": {"source": "fake", "seq_len": 128, "fake_vocab_size": 64,
                                            "fake_prompt_len": 6},
                                   "inference": {"vllm": {"server_backend": "offline", "reasoning_parser": None,
                                                          "tool_call_parser": None}},
                                   "lora": None, "output_dir": str(tmp_path / "out")})
    tok = CharTokenizer()
    c = TestClient(build_app(cfg, engine=_StubEngine(tok, "yes. STOP ignored tail")))
    ch = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "q"}],
                                              "stop": [" STOP"]}).json()
    assert ch["choices"][0]["message"]["content"] == "yes." and ch["choices"][0]["finish_reason"] == "stop"
    assert tok.decode(ch["choices"][0]["token_ids"]) == "yes. STOP"
    assert ch["usage"]["completion_tokens"] == len(ch["choices"][0]["token_ids"])


def test_concurrent_requests_share_generator_batches():
    import threading as _th
    import time as _time

    from wavelet_b200.inference.engine import Completion
    from wavelet_b200.inference.server import RequestBatcher

    calls = []

    def run(prompts, settings):
        calls.append((len(prompts), settings["temperature"]))
        _time.sleep(0.05)
        return [Completion(i, k, p, [p[0], k], [-0.1, -0.2], "stop") for i, p in enumerate(prompts)
                for k in range(settings.get("n") or 1)]

    # min_size 6: the worker waits (up to max_wait_seconds) until the six requests are queued
    b = RequestBatcher(run, wait_seconds=0.0, max_wait_seconds=5.0, min_size=6, max_size=None)
    out = {}

    def client(i, temp):
        out[i] = b.submit([[100 + i], [200 + i]], {"temperature": temp, "n": 2})

    ths = [_th.Thread(target=client, args=(i, 1.0 if i < 4 else 0.5)) for i in range(6)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    # two generator calls: one per sampling setting, each holding every request with it
    assert sorted(calls) == [(4, 0.5), (8, 1.0)]
    for i in range(6):
        assert [(c.prompt_index, c.sample_index, c.token_ids[0]) for c in out[i]] == \
            [(0, 0, 100 + i), (0, 1, 100 + i), (1, 0, 200 + i), (1, 1, 200 + i)]
    # max_size bounds the requests per batch; an error reaches every waiter of its batch
    calls.clear()
    b2 = RequestBatcher(run, wait_seconds=0.05, max_size=2)
    ths = [_th.Thread(target=client, args=(i, 1.0)) for i in range(4)]
    b = b2
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    assert all(n <= 4 for n, _ in calls)

    def boom(prompts, settings):
        raise RuntimeError("generator failed")

    b3 = RequestBatcher(boom, wait_seconds=0.0)
    with pytest.raises(RuntimeError, match="generator failed"):
        b3.submit([[1]], {"temperature": 1.0})
