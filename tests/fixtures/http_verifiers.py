"""A stand-in ``verifiers`` package for an end-to-end test: its environment
calls the OpenAI chat-completions-with-tokens route of the inference server it
is given, like a real verifiers environment, and scores the sampled tokens."""

import asyncio
import json
import urllib.request


class ClientConfig:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def RolloutInput(**kw):  # noqa: N802 - the package's name
    return dict(kw)


class _Rows:
    def __init__(self, rows):
        self.rows = rows

    def to_list(self):
        return [dict(r) for r in self.rows]


class HttpEnv:
    requires_group_scoring = False

    def __init__(self, n=3):
        self.rows = [{"prompt": [{"role": "user", "content": f"count {i}"}], "example_id": i} for i in range(n)]

    def set_kwargs(self, **kw):
        self.kwargs = kw

    def get_dataset(self, n=-1, seed=None):
        return _Rows(self.rows)

    def _post(self, url, body):
        req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=60) as r:
            return json.loads(r.read())

    async def run_rollout(self, inp, client, model, sampling_args, max_retries=0, state_columns=None):
        ex = int(inp["example_id"])
        prompt = [10 + ex, 11, 12]
        body = {"model": model, "messages": inp["prompt"], "tokens": prompt, "max_tokens": 4, "logprobs": True,
                "temperature": sampling_args.get("temperature", 1.0), **sampling_args.get("extra_body", {})}
        out = await asyncio.to_thread(self._post, client.api_base_url + "/chat/completions/tokens", body)
        ch = out["choices"][0]
        ids = ch["token_ids"]
        lps = [x["logprob"] for x in ch["logprobs"]["content"]]
        reward = sum(t % 2 == 0 for t in ids) / max(len(ids), 1)
        return {"example_id": ex, "reward": reward, "sampling_args": dict(sampling_args), "is_truncated": False,
                "trajectory": [{"prompt": inp["prompt"], "completion": [{"role": "assistant", "content": "x"}],
                                "tokens": {"prompt_ids": out["prompt_token_ids"], "completion_ids": ids,
                                           "completion_mask": [1] * len(ids), "completion_logprobs": lps}}]}


def load_environment(env_id, **args):
    return HttpEnv(**args)
