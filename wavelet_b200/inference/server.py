"""``wavelet inference-server``: the native generator behind HTTP.

Routes (the reference's inference server surface, inference/server.py:693-1036
and native_server.py:92-215):

    GET  /health, /liveness, /debug/state, /v1/models, /metrics
    POST /pause, /resume, /sleep, /wake
    POST /load_policy            {"policy_dir": ..., "step": N}
    POST /init_broadcaster       device weight transfer group (flat_v1 protocol)
    POST /annotate               {"records": [RLExample payloads]} -> annotated records
    POST /score                  teacher-forced log-probs of given token sequences
    POST /v1/completions         {"prompt_token_ids" | "prompt", sampling...}
    POST /v1/chat/completions[/tokens], /chat/completions/tokens
                                 reasoning / tool calls split by the configured
                                 parsers (inference/parsers.py), max_tokens
                                 fitted to the context
    POST /tokenize, /v1/tokenize

Concurrent generation requests are collected into shared generator batches
(``RequestBatcher``, ``inference.vllm.openai_batch_*``); a gate that
``/pause`` closes holds new requests while a policy is being loaded.
"""

from __future__ import annotations

import json
import sys
import threading
import time
import uuid
from contextlib import contextmanager
from pathlib import Path
from types import SimpleNamespace
from typing import Any

from ..configs.config import RLConfig
from ..data.rl import example_from_payload, example_to_payload
from ..utils.config import load_config
from .parsers import ChatOutputParser

CONTEXT_FIT_SAFETY_TOKENS = 16  # tokens kept free when a request's max_tokens is fitted to the context


def apply_stop_strings(tok, ids: list[int], logprobs: list[float], stops) -> tuple[list[int], list[float], str, bool]:
    """A completion cut at the first OpenAI ``stop`` string: the tokens up to
    the one that completes it (their log-probs kept), the text before it, and
    whether a stop string was found.  The generator samples whole completions,
    so the cut is made afterwards; tokens sampled before the stop point do not
    depend on the ones after it."""
    text = tok.decode(ids)
    stops = [stops] if isinstance(stops, str) else [x for x in (stops or []) if x]
    hits = [(text.find(x), x) for x in stops if x in text]
    if not hits:
        return ids, logprobs, text, False
    pos, stop = min(hits)
    lo, hi = 1, len(ids)  # smallest prefix whose text contains the stop string
    while lo < hi:
        mid = (lo + hi) // 2
        if stop in tok.decode(ids[:mid]):
            hi = mid
        else:
            lo = mid + 1
    return ids[:lo], logprobs[:lo], text[:pos], True


class RequestBatcher:
    """Concurrent generation requests run as one generator batch
    (``inference.vllm.openai_batch_*``; ref inference/engine.py:958-1000).

    The worker takes the first waiting request, waits ``wait_seconds`` for
    others, keeps waiting up to ``max_wait_seconds`` while fewer than
    ``min_size`` are queued, takes at most ``max_size`` requests, and runs the
    requests with equal sampling settings as one ``run(prompts, settings)``
    call; every request gets its own completions back (``prompt_index``
    relative to its own prompts).  An error fails every request of the
    batch."""

    def __init__(self, run, *, wait_seconds: float = 0.01, min_size: int = 1, max_wait_seconds: float = 0.01,
                 max_size: int | None = None):
        self.run = run
        self.wait, self.min_size = wait_seconds, min_size
        self.max_wait = max(wait_seconds, max_wait_seconds)
        self.max_size = max_size
        self._queue: list[dict[str, Any]] = []
        self._cv = threading.Condition()
        self._thread = threading.Thread(target=self._loop, name="wavelet-batcher", daemon=True)
        self._thread.start()
        self.batches = 0  # generator calls made (for tests and metrics)

    def submit(self, prompts: list[list[int]], settings: dict[str, Any]) -> list[Any]:
        req = {"prompts": prompts, "settings": settings, "done": threading.Event(), "result": None, "error": None}
        with self._cv:
            self._queue.append(req)
            self._cv.notify_all()
        req["done"].wait()
        if req["error"] is not None:
            raise req["error"]
        return req["result"]

    def _take(self) -> list[dict[str, Any]]:
        t0 = time.perf_counter()
        if self.wait > 0:
            self._cv.wait(timeout=self.wait)
        while len(self._queue) < self.min_size:
            left = t0 + self.max_wait - time.perf_counter()
            if left <= 0:
                break
            self._cv.wait(timeout=left)
        n = len(self._queue) if self.max_size is None else min(self.max_size, len(self._queue))
        batch, self._queue = self._queue[:n], self._queue[n:]
        return batch

    def _loop(self) -> None:
        from dataclasses import replace

        while True:
            with self._cv:
                while not self._queue:
                    self._cv.wait()
                batch = self._take()
            groups: dict[str, list[dict[str, Any]]] = {}
            for r in batch:
                groups.setdefault(json.dumps(r["settings"], sort_keys=True, default=str), []).append(r)
            for reqs in groups.values():
                try:
                    prompts, offsets = [], []
                    for r in reqs:
                        offsets.append(len(prompts))
                        prompts += r["prompts"]
                    comps = self.run(prompts, reqs[0]["settings"])
                    self.batches += 1
                    for r, o in zip(reqs, offsets):
                        mine = [c for c in comps if o <= c.prompt_index < o + len(r["prompts"])]
                        r["result"] = [replace(c, prompt_index=c.prompt_index - o) for c in mine]
                except BaseException as exc:  # noqa: BLE001 - every waiter learns of it
                    for r in reqs:
                        r["error"] = exc
                for r in reqs:
                    r["done"].set()


class GenerationGate:
    def __init__(self):
        self._cv = threading.Condition()
        self._paused = False
        self._active = 0

    @contextmanager
    def generation(self):
        with self._cv:
            while self._paused:
                self._cv.wait()
            self._active += 1
        try:
            yield
        finally:
            with self._cv:
                self._active -= 1
                self._cv.notify_all()

    def pause(self, wait: bool = True):
        with self._cv:
            self._paused = True
            while wait and self._active:
                self._cv.wait()

    def resume(self):
        with self._cv:
            self._paused = False
            self._cv.notify_all()

    @property
    def paused(self) -> bool:
        return self._paused

    @property
    def active(self) -> int:
        return self._active


def build_app(config: RLConfig, engine=None):
    from fastapi import FastAPI, HTTPException

    from ..data.tokenizer import tokenizer_for
    from .policy import NativePolicyInferenceEngine

    tok = tokenizer_for(config.model)
    if engine is None:
        engine = NativePolicyInferenceEngine(config, tokenizer=tok)
        engine.setup()
        if config.policy_transfer.type == "nccl":
            import os

            engine.attach_device_receiver(int(os.environ.get("WAVELET_INFERENCE_REPLICA", "0")))
    gate = GenerationGate()
    vb = config.inference.vllm

    def _run_batch(prompts, ov):
        with lock:
            return engine.generate_ids(prompts, ov)

    # concurrent completion requests share generator batches
    batcher = RequestBatcher(_run_batch, wait_seconds=vb.openai_batch_wait_seconds, min_size=vb.openai_batch_min_size,
                             max_wait_seconds=vb.openai_batch_max_wait_seconds, max_size=vb.openai_batch_max_size)
    app = FastAPI(title="wavelet inference server")
    app.state.engine = engine
    state: dict[str, Any] = {"started_at": time.time(), "requests": 0, "generated_tokens": 0, "sleeping": False}
    lock = threading.Lock()

    @app.get("/health")
    def health():
        return {"status": "ok"}

    @app.get("/liveness")
    def liveness():
        return {"status": "alive", "paused": gate.paused, "sleeping": state["sleeping"]}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": config.model.name, "object": "model", "owned_by": "wavelet"}]}

    @app.get("/debug/state")
    def debug_state():
        g = engine.generator
        return {"policy_step": engine.policy_step, "paused": gate.paused, **state,
                "kv_cache_usage": g.kv_usage() if g is not None else None,
                "num_blocks": g.num_blocks if g is not None else None}

    @app.get("/metrics")
    def metrics():
        g = engine.generator
        usage = g.kv_usage() if g is not None else 0.0
        active = gate.active  # requests inside the gate: one generates at a time, the rest wait for it
        lines = [
            f"wavelet:kv_cache_usage_perc {usage}",
            f"wavelet:num_requests_running {min(active, 1)}",
            f"wavelet:num_requests_waiting {max(active - 1, 0)}",
            f"wavelet:generation_tokens_total {state['generated_tokens']}",
            f"wavelet:requests_total {state['requests']}",
        ]
        from fastapi.responses import PlainTextResponse

        return PlainTextResponse("\n".join(lines) + "\n")

    @app.post("/pause")
    def pause():
        gate.pause()
        return {"status": "paused"}

    @app.post("/resume")
    def resume():
        gate.resume()
        return {"status": "resumed"}

    @app.post("/sleep")
    def sleep():
        gate.pause()
        engine.sleep()
        state["sleeping"] = True
        return {"status": "sleeping"}

    @app.post("/wake")
    def wake(payload: dict[str, Any] | None = None):
        engine.wake(tags=(payload or {}).get("tags"))
        state["sleeping"] = False
        gate.resume()
        return {"status": "awake"}

    @app.post("/load_policy")
    def load_policy(payload: dict[str, Any]):
        step = int(payload["step"])
        pdir = payload.get("policy_dir")
        with lock:
            engine.load_policy(Path(pdir) if pdir else None, step=step)
        return {"status": "loaded", "policy_step": step}

    @app.post("/init_broadcaster")
    def init_broadcaster(payload: dict[str, Any] | None = None):
        """Device transfer setup: the receive slots of this generator (peer
        path) or the NCCL group coordinates of the fallback."""
        rec = getattr(engine, "device_receiver", None)
        if rec is None and config.policy_transfer.type == "nccl" and hasattr(engine, "attach_device_receiver"):
            rec = engine.attach_device_receiver(int((payload or {}).get("index", 0)))
        if rec is None:
            return {"status": "off"}
        pt = config.policy_transfer
        out = {"status": "ok", "protocols": ["peer_v1", "flat_v1"] if rec.peer is not None else ["flat_v1"],
               "nccl": {"host": pt.nccl_host, "port": pt.nccl_port, "rank": pt.nccl_rank_offset + rec.index,
                        "world_size": 1 + pt.nccl_inference_world_size}}
        if rec.peer is not None:
            out["peer"] = {"receiver": str(rec.peer.path), "slots": rec.peer.slots, "epochs": rec.peer.epochs()}
        return out

    @app.post("/annotate")
    def annotate(payload: dict[str, Any]):
        with gate.generation(), lock:
            recs = [example_from_payload(r) for r in payload["records"]]
            out = engine.annotate(recs)
        state["requests"] += 1
        state["generated_tokens"] += sum(len((r.metadata or {}).get("completion_ids", [])) for r in out)
        return {"records": [example_to_payload(r) for r in out], "policy_step": engine.policy_step}

    @app.post("/score")
    def score(payload: dict[str, Any]):
        with gate.generation(), lock:
            lps = engine.score(payload["sequences"], payload["prompt_lens"], float(payload.get("temperature", 1.0)))
        return {"logprobs": lps}

    def _complete(prompts: list[list[int]], payload: dict[str, Any]) -> list[Any]:
        # OpenAI fields and the vLLM-style extras clients send in extra_body (top_k, min_p, min_tokens,
        # stop_token_ids), merged into the request body by the OpenAI client
        ov = {"temperature": payload.get("temperature"), "top_p": payload.get("top_p"),
              "top_k": payload.get("top_k"), "min_p": payload.get("min_p"),
              "max_tokens": payload.get("max_completion_tokens") or payload.get("max_tokens"),
              "min_tokens": payload.get("min_tokens"), "stop_token_ids": payload.get("stop_token_ids"),
              "n": payload.get("n"), "seed": payload.get("seed")}
        with gate.generation():
            return batcher.submit(prompts, ov)

    @app.post("/v1/completions")
    def completions(payload: dict[str, Any]):
        if "prompt_token_ids" in payload:
            prompts = payload["prompt_token_ids"]
            prompts = [prompts] if prompts and isinstance(prompts[0], int) else prompts
        else:
            p = payload["prompt"]
            prompts = [tok.encode(x) for x in ([p] if isinstance(p, str) else p)]
        comps = _complete(prompts, payload)
        if payload.get("stop"):
            cut = []
            for c in comps:
                ids_c, lps_c, _, hit = apply_stop_strings(tok, c.token_ids, c.logprobs, payload["stop"])
                cut.append(SimpleNamespace(token_ids=ids_c, logprobs=lps_c, prompt_index=c.prompt_index,
                                           finish_reason="stop" if hit else c.finish_reason))
            comps = cut
        body = {"object": "text_completion", "model": config.model.name, "policy_step": engine.policy_step,
                "choices": [{"index": i, "prompt_index": c.prompt_index, "token_ids": c.token_ids,
                             "logprobs": {"token_logprobs": c.logprobs}, "text": tok.decode(c.token_ids),
                             "finish_reason": c.finish_reason} for i, c in enumerate(comps)]}
        if payload.get("stream"):  # one chunk per choice, then the end marker
            return _sse({**body, "choices": [ch]} for ch in body["choices"])
        return body

    vcfg = config.inference.vllm
    out_parser = ChatOutputParser.for_model(config.model.name, vcfg.reasoning_parser, vcfg.tool_call_parser)

    def _max_model_len() -> int:
        g = getattr(engine, "generator", None)
        return int(getattr(g, "max_model_len", None) or vcfg.max_model_len or config.data.seq_len)

    def _chat(payload: dict[str, Any]):
        """OpenAI chat completion.  ``tokens`` (the ``/chat/completions/tokens``
        routes) is the rendered prompt; otherwise ``messages`` is rendered with
        the chat template, with ``tools`` and ``chat_template_kwargs``.  The
        completion is split into reasoning, content and tool calls by the
        configured parsers, and a request whose prompt plus ``max_tokens``
        overruns the context gets its ``max_tokens`` fitted
        (ref inference/server.py:186-220, 482-520)."""
        kwargs = dict(payload.get("chat_template_kwargs") or {})
        tools = payload.get("tools") or None
        if payload.get("tokens") is not None:
            ids = [int(t) for t in payload["tokens"]]
        else:
            extra = {"tools": tools} if tools else {}
            ids = tok.apply_chat_template(payload["messages"], tokenize=True, add_generation_prompt=True,
                                          **extra, **kwargs)
            ids = list(ids["input_ids"] if isinstance(ids, dict) else ids)
        limit = _max_model_len()
        if len(ids) >= limit:
            raise HTTPException(status_code=400, detail=f"This model's maximum context length is {limit} tokens. "
                                                        f"However, your request has {len(ids)} input tokens.")
        req = dict(payload)
        asked = payload.get("max_completion_tokens") or payload.get("max_tokens") \
            or config.inference.sampling.max_completion_tokens or 256
        room = max(limit - len(ids) - CONTEXT_FIT_SAFETY_TOKENS, 1)
        req["max_completion_tokens"] = min(int(asked), room)
        comps = _complete([ids], req)
        choices = []
        for i, c in enumerate(comps):
            if payload.get("stop"):
                ids_c, lps_c, text, hit = apply_stop_strings(tok, c.token_ids, c.logprobs, payload["stop"])
                c = SimpleNamespace(token_ids=ids_c, logprobs=lps_c, finish_reason="stop" if hit else c.finish_reason,
                                    prompt_index=getattr(c, "prompt_index", 0))
            else:
                text = tok.decode(c.token_ids)
            parsed = out_parser.parse(text, tools=tools,
                                      tool_choice=payload.get("tool_choice", "auto"),
                                      include_reasoning=bool(payload.get("include_reasoning", True)),
                                      chat_template_kwargs=kwargs)
            finish = "tool_calls" if parsed.tool_calls and c.finish_reason == "stop" else c.finish_reason
            choices.append({"index": i, "message": parsed.message(), "token_ids": c.token_ids,
                            "logprobs": {"content": [{"token": f"token_id:{t}", "token_id": t, "logprob": lp}
                                                     for t, lp in zip(c.token_ids, c.logprobs)]},
                            "finish_reason": finish})
        n_out = sum(len(ch["token_ids"]) for ch in choices)
        body = {"object": "chat.completion", "model": config.model.name, "prompt_token_ids": ids,
                "choices": choices,
                "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out, "total_tokens": len(ids) + n_out}}
        if payload.get("stream"):
            return _sse(_chat_chunks(body))
        return body

    def _chat_chunks(body: dict[str, Any]):
        """``chat.completion.chunk`` events of a finished completion: the role,
        the reasoning, the content, the tool calls, then the finish reason
        (the generator returns whole completions, so the stream follows it)."""
        rid = "chatcmpl-" + uuid.uuid4().hex[:24]
        base = {"id": rid, "object": "chat.completion.chunk", "created": int(time.time()), "model": body["model"]}
        for ch in body["choices"]:
            i, msg = ch["index"], ch["message"]
            yield {**base, "choices": [{"index": i, "delta": {"role": "assistant"}, "finish_reason": None}]}
            if msg.get("reasoning_content"):
                yield {**base, "choices": [{"index": i, "delta": {"reasoning_content": msg["reasoning_content"]},
                                            "finish_reason": None}]}
            if msg.get("content"):
                yield {**base, "choices": [{"index": i, "delta": {"content": msg["content"]}, "finish_reason": None,
                                            "logprobs": ch["logprobs"]}]}
            for k, tc in enumerate(msg.get("tool_calls") or []):
                yield {**base, "choices": [{"index": i, "delta": {"tool_calls": [{"index": k, **tc}]},
                                            "finish_reason": None}]}
            yield {**base, "choices": [{"index": i, "delta": {}, "finish_reason": ch["finish_reason"],
                                        "token_ids": ch["token_ids"]}]}
        yield {**base, "choices": [], "usage": body["usage"], "prompt_token_ids": body["prompt_token_ids"]}

    def _sse(events):
        from fastapi.responses import StreamingResponse

        def gen():
            for e in events:
                yield "data: " + json.dumps(e) + "\n\n"
            yield "data: [DONE]\n\n"

        return StreamingResponse(gen(), media_type="text/event-stream")

    app.post("/v1/chat/completions")(_chat)
    app.post("/v1/chat/completions/tokens")(_chat)
    app.post("/chat/completions/tokens")(_chat)

    def _tokenize(payload: dict[str, Any]):
        if "messages" in payload:
            ids = tok.apply_chat_template(payload["messages"], tokenize=True,
                                          add_generation_prompt=bool(payload.get("add_generation_prompt", True)))
            ids = list(ids["input_ids"] if isinstance(ids, dict) else ids)
        else:
            ids = tok.encode(payload.get("prompt", ""))
        return {"tokens": ids, "count": len(ids)}

    app.post("/tokenize")(_tokenize)
    app.post("/v1/tokenize")(_tokenize)
    app.state.engine = engine
    app.state.gate = gate
    app.state.batcher = batcher
    return app


class InProcessServer:
    """The OpenAI routes of ``build_app`` served from a thread of this
    process (integrated RL with verifiers-package environments: the
    environments call the generator that shares the trainer's process)."""

    def __init__(self, config: RLConfig, engine, host: str = "127.0.0.1", port: int = 0):
        import socket

        import uvicorn

        if port == 0:
            with socket.socket() as sk:
                sk.bind((host, 0))
                port = sk.getsockname()[1]
        self.host, self.port = host, port
        self.app = build_app(config, engine=engine)
        self._server = uvicorn.Server(uvicorn.Config(self.app, host=host, port=port, log_level="warning"))
        self._thread = threading.Thread(target=self._server.run, name="wavelet-openai", daemon=True)

    @property
    def base_url(self) -> str:
        return f"http://{self.host}:{self.port}/v1"

    def start(self, timeout: float = 30.0) -> "InProcessServer":
        self._thread.start()
        t0 = time.time()
        while not self._server.started:
            if not self._thread.is_alive() or time.time() - t0 > timeout:
                raise RuntimeError(f"the in-process OpenAI server did not start on {self.host}:{self.port}")
            time.sleep(0.01)
        return self

    def close(self) -> None:
        self._server.should_exit = True
        self._thread.join(timeout=10)


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config(RLConfig, argv)
    if cfg.inference.vllm.tensor_parallel_size > 1:  # one replica over a torchrun group of processes
        from .tp_server import run_tp_server

        return run_tp_server(cfg)
    import uvicorn

    app = build_app(cfg)
    try:
        uvicorn.run(app, host=cfg.inference.http.host, port=cfg.inference.http.port, log_level="warning")
    finally:
        app.state.engine.close()  # releases the device policy receive slots
    return 0


if __name__ == "__main__":
    sys.exit(main())
