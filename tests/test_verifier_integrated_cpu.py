"""End to end on the CPU: integrated RL with a verifiers-package environment.
The runner serves its own generator on an in-process OpenAI server, the
(stand-in) environment samples through the chat-completions-with-tokens route,
and its rollouts train the policy for two steps."""

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_integrated_rl_with_a_verifiers_environment(tmp_path):
    pkg = tmp_path / "site" / "verifiers"
    pkg.mkdir(parents=True)
    shutil.copy(ROOT / "tests" / "fixtures" / "http_verifiers.py", pkg / "__init__.py")
    cfg = tmp_path / "rl.yaml"
    cfg.write_text(f"""model:
  name: tiny
  random_init: true
data:
  source: fake
  seq_len: 128
algo:
  type: grpo
reward:
  mode: passthrough
orchestrator:
  verifier_env_id: http-env
  verifier_env_args: {{n: 3}}
  examples_per_step: 2
  rollouts_per_example: 3
  filter_zero_advantage: false
inference:
  sampling:
    max_completion_tokens: 4
lora: null
max_steps: 2
output_dir: {tmp_path / 'out'}
""")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1",
           "PYTHONPATH": os.pathsep.join([str(tmp_path / "site"), str(ROOT), os.environ.get("PYTHONPATH", "")])}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "rl", "@", str(cfg)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(l) for l in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2]
    assert rows[0]["verifier/rollouts"] == 6.0 and "progress/tokens" in rows[0]
    batch = [json.loads(l) for l in (tmp_path / "out" / "rollouts" / "step-000000" / "rollouts.jsonl")
             .read_text().splitlines()]
    assert len(batch) == 6 and all(b["metadata"]["reward_source"] == "verifier" for b in batch)
    # sampled tokens are trained, with their log-probs (up to 4: a sampled end token stops early)
    assert all(1 <= sum(b["loss_mask"]) <= 4 and len(b["inference_logprobs"]) == sum(b["loss_mask"]) for b in batch)
