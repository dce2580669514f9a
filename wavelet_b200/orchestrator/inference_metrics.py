"""Engine load scraping for the concurrency controller (reference
orchestrator/inference_metrics.py:40-136).

Reads either a Prometheus text exposition (``/metrics``; vLLM-style names
``vllm:gpu_cache_usage_perc`` / ``vllm:kv_cache_usage_perc``,
``vllm:num_requests_running``, ``vllm:num_requests_waiting``,
``vllm:num_preemptions_total``, ``vllm:generation_tokens_total``, or the
native server's ``wavelet:`` equivalents) or the native ``/debug/state``
JSON, into an ``EngineLoad``.
"""

from __future__ import annotations

import json
import re
import urllib.request

from .concurrency import EngineLoad

_LINE = re.compile(r'^([a-zA-Z_:][a-zA-Z0-9_:]*)(\{[^}]*\})?\s+([-+0-9.eEinfNa]+)')
_NAMES = {
    "kv": ("vllm:kv_cache_usage_perc", "vllm:gpu_cache_usage_perc", "wavelet:kv_cache_usage_perc"),
    "running": ("vllm:num_requests_running", "wavelet:num_requests_running"),
    "waiting": ("vllm:num_requests_waiting", "wavelet:num_requests_waiting"),
    "preemptions": ("vllm:num_preemptions_total", "vllm:num_preemptions"),
    "gen_tokens": ("vllm:generation_tokens_total", "wavelet:generation_tokens_total"),
}


def parse_prometheus(text: str) -> dict[str, float]:
    """Sum every sample of a metric name over its label sets."""
    out: dict[str, float] = {}
    for line in text.splitlines():
        if not line or line.startswith("#"):
            continue
        m = _LINE.match(line.strip())
        if not m:
            continue
        try:
            v = float(m.group(3))
        except ValueError:
            continue
        out[m.group(1)] = out.get(m.group(1), 0.0) + v
    return out


class EngineMetricsScraper:
    def __init__(self):
        self._prev_preempt: dict[str, float] = {}

    def from_prometheus(self, text: str, replica: str = "0") -> EngineLoad:
        vals = parse_prometheus(text)

        def pick(key: str) -> float:
            for n in _NAMES[key]:
                if n in vals:
                    return vals[n]
            return 0.0

        pre = pick("preemptions")
        delta = pre - self._prev_preempt.get(replica, pre)
        self._prev_preempt[replica] = pre
        return EngineLoad(kv_cache_usage=pick("kv"), running=int(pick("running")), waiting=int(pick("waiting")),
                          preemptions_delta=int(max(0, delta)))

    @staticmethod
    def from_native_state(state: dict) -> EngineLoad:
        return EngineLoad(kv_cache_usage=float(state.get("kv_cache_usage") or 0.0),
                          running=int(state.get("running") or 0), waiting=int(state.get("waiting") or 0))

    def scrape(self, base_url: str, timeout: float = 5.0) -> EngineLoad:
        try:
            with urllib.request.urlopen(base_url + "/metrics", timeout=timeout) as r:
                return self.from_prometheus(r.read().decode(), base_url)
        except Exception:  # native server: JSON state instead
            with urllib.request.urlopen(base_url + "/debug/state", timeout=timeout) as r:
                return self.from_native_state(json.loads(r.read()))
