"""HTTP client engine: drives one or more ``inference-server`` replicas.

``load_policy`` pauses every replica, loads the snapshot, and resumes;
``annotate`` splits the records round-robin across replicas, retrying a
failed request on the next replica (inference/engine.py:292-669 of the
reference).
"""

from __future__ import annotations

import json
import time
import urllib.error
import urllib.request
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any

from ..data.rl import RLExample, example_from_payload, example_to_payload
from .policy import PolicyInferenceEngine


def endpoints(cfg) -> list[str]:
    h = cfg.inference.http
    if h.ports is not None:
        hosts = h.hosts or [h.host] * len(h.ports)
        return [f"http://{a}:{p}" for a, p in zip(hosts, h.ports)]
    hosts = h.hosts or [h.host]
    return [f"http://{a}:{h.port}" for a in hosts]


def http_json(url: str, payload: dict | None = None, timeout: float = 30.0) -> dict[str, Any]:
    data = None if payload is None else json.dumps(payload).encode()
    req = urllib.request.Request(url, data=data, method="GET" if payload is None else "POST",
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        body = r.read()
        return json.loads(body) if body else {}


def wait_healthy(urls: list[str], timeout: float, poll: float = 1.0, probe_timeout: float = 5.0) -> None:
    """Poll every server's /health until all answer; each probe waits at most
    ``probe_timeout`` (inference.http.liveness_timeout_seconds)."""
    t0 = time.monotonic()
    pending = list(urls)
    while pending:
        still = []
        for u in pending:
            try:
                http_json(u + "/health", timeout=min(probe_timeout, timeout))
            except (urllib.error.URLError, OSError, ValueError):
                still.append(u)
        pending = still
        if pending:
            if time.monotonic() - t0 > timeout:
                raise TimeoutError(f"inference servers not healthy after {timeout}s: {pending}")
            time.sleep(poll)


class HTTPPolicyInferenceEngine(PolicyInferenceEngine):
    concurrent_generate = True  # the servers batch concurrent requests
    concurrent_policy_load = True  # a weight load pauses the servers' generation itself

    def __init__(self, config):
        super().__init__(config)
        self.urls = endpoints(config)
        self.rr = 0

    def setup(self) -> None:
        h = self.config.inference.http
        wait_healthy(self.urls, h.startup_timeout_seconds, probe_timeout=h.liveness_timeout_seconds)
        for u in self.urls:
            http_json(u + "/v1/models", timeout=h.request_timeout_seconds)

    def load_policy(self, policy_dir: Path, *, step: int) -> None:
        h = self.config.inference.http
        for u in self.urls:
            http_json(u + "/pause", {}, timeout=h.request_timeout_seconds)
        try:
            for u in self.urls:
                http_json(u + "/load_policy", {"policy_dir": str(policy_dir) if policy_dir else None, "step": step},
                          timeout=h.request_timeout_seconds)
        finally:
            for u in self.urls:
                http_json(u + "/resume", {}, timeout=h.request_timeout_seconds)
        self.policy_step = step

    def annotate(self, records: list[RLExample]) -> list[RLExample]:
        if not records:
            return []
        n = len(self.urls)
        shards = [records[i::n] for i in range(n)]
        h = self.config.inference.http

        def run(i: int):
            last = None
            for attempt in range(n):
                u = self.urls[(i + attempt) % n]
                try:
                    r = http_json(u + "/annotate", {"records": [example_to_payload(x) for x in shards[i]]},
                                  timeout=h.request_timeout_seconds)
                    return [example_from_payload(x) for x in r["records"]]
                except (urllib.error.URLError, OSError, ValueError) as e:
                    last = e
            raise RuntimeError(f"annotate failed on every replica: {last}")

        with ThreadPoolExecutor(max_workers=n) as ex:
            parts = list(ex.map(run, range(n)))
        out: list[RLExample] = [None] * len(records)  # type: ignore[list-item]
        for i, part in enumerate(parts):
            for j, r in enumerate(part):
                out[i + j * n] = r
        return out

    def sleep(self) -> None:
        for u in self.urls:
            http_json(u + "/sleep", {}, timeout=self.config.inference.http.request_timeout_seconds)

    def wake(self, *, tags: list[str] | None = None) -> None:
        for u in self.urls:
            http_json(u + "/wake", {"tags": tags}, timeout=self.config.inference.http.request_timeout_seconds)

    def kv_cache_usage(self) -> float:
        vals = []
        for u in self.urls:
            try:
                vals.append(float(http_json(u + "/debug/state", timeout=5.0).get("kv_cache_usage") or 0.0))
            except (urllib.error.URLError, OSError, ValueError):
                pass
        return max(vals) if vals else 0.0
