"""``python -m wavelet_b200.tools.chat``: chat with a running
OpenAI-compatible server (``wavelet_b200.inference.server`` or any other),
interactively or for one ``--prompt`` (reference scripts/chat.py).

The model id defaults to the first entry of ``GET {base}/models``; the API key
is read from the environment variable named by ``--api-key-var``.  The
conversation history is resent with every turn; an assistant message with
tool calls but no text is shown as its JSON.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import urllib.error
import urllib.request
from typing import Any


def request_json(url: str, api_key: str | None = None, payload: dict | None = None, timeout: float = 300.0) -> dict:
    headers = {"Accept": "application/json"}
    if api_key:
        headers["Authorization"] = f"Bearer {api_key}"
    body = None
    if payload is not None:
        headers["Content-Type"] = "application/json"
        body = json.dumps(payload).encode()
    req = urllib.request.Request(url, data=body, headers=headers, method="POST" if body is not None else "GET")
    try:
        with urllib.request.urlopen(req, timeout=timeout) as resp:
            out = json.loads(resp.read().decode())
    except urllib.error.HTTPError as e:
        raise RuntimeError(f"request to {url} failed with HTTP {e.code}: {e.read().decode(errors='replace')}") from e
    except urllib.error.URLError as e:
        raise RuntimeError(f"cannot reach the inference server at {url}: {e.reason}") from e
    if not isinstance(out, dict):
        raise TypeError("the server answered with a non-object JSON value")
    return out


def first_model(base: str, api_key: str | None, timeout: float) -> str:
    data = request_json(f"{base}/models", api_key, None, timeout).get("data")
    if not isinstance(data, list) or not data or not isinstance(data[0], dict) or not isinstance(data[0].get("id"), str):
        raise RuntimeError("the server listed no models at /models")
    return data[0]["id"]


def reply_text(resp: dict[str, Any]) -> str:
    choices = resp.get("choices")
    if not isinstance(choices, list) or not choices or not isinstance(choices[0], dict):
        raise RuntimeError("the chat completion has no choices")
    msg = choices[0].get("message")
    if not isinstance(msg, dict):
        raise TypeError("the chat completion choice has no message")
    if isinstance(msg.get("content"), str) and msg["content"]:
        return msg["content"]
    if msg.get("tool_calls"):
        return json.dumps(msg["tool_calls"], ensure_ascii=False, indent=2)
    return ""


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Chat with an OpenAI-compatible server.")
    ap.add_argument("--base-url", default="http://127.0.0.1:8000/v1")
    ap.add_argument("--model")
    ap.add_argument("--api-key-var", default="OPENAI_API_KEY")
    ap.add_argument("--system")
    ap.add_argument("--prompt", help="send one prompt and exit")
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--max-completion-tokens", type=int)
    ap.add_argument("--reasoning-effort", choices=["minimal", "low", "medium", "high"])
    ap.add_argument("--timeout", type=float, default=300.0)
    a = ap.parse_args(argv)
    base = a.base_url.rstrip("/")
    key = os.environ.get(a.api_key_var)
    model = a.model or first_model(base, key, a.timeout)
    history: list[dict[str, str]] = [{"role": "system", "content": a.system}] if a.system else []

    def turn(text: str) -> None:
        history.append({"role": "user", "content": text})
        payload: dict[str, Any] = {"model": model, "messages": history, "temperature": a.temperature}
        if a.max_completion_tokens is not None:
            payload["max_completion_tokens"] = a.max_completion_tokens
        if a.reasoning_effort is not None:
            payload["reasoning_effort"] = a.reasoning_effort
        out = reply_text(request_json(f"{base}/chat/completions", key, payload, a.timeout))
        history.append({"role": "assistant", "content": out})
        print(out, flush=True)

    if a.prompt is not None:
        turn(a.prompt)
        return 0
    print(f"Connected to {model}. /exit quits.")
    while True:
        try:
            line = input("you> ")
        except (EOFError, KeyboardInterrupt):
            print()
            return 0
        if line.strip().lower() in ("/exit", "/quit"):
            return 0
        if line.strip():
            turn(line)


if __name__ == "__main__":
    sys.exit(main())
