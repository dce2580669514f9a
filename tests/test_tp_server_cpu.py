"""A tensor-parallel inference server replica on 2 gloo CPU processes
(torchrun): rank 0 serves HTTP and announces every engine call to rank 1;
greedy completions equal those of the single-process server, and a policy
exported by the trainer loads into both ranks' parts."""

import json
import os
import socket
import subprocess
import sys
import time
import urllib.request
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(tmp: Path, name: str, port: int, tp: int) -> Path:
    p = tmp / f"{name}.yaml"
    p.write_text(f"""model:
  name: tiny
  random_init: true
seed: 3
data:
  source: fake
  seq_len: 128
inference:
  vllm:
    tensor_parallel_size: {tp}
    max_num_seqs: 8
    max_model_len: 128
  http:
    port: {port}
lora: null
output_dir: {tmp / name}
""")
    return p


def _post(port: int, route: str, payload: dict) -> dict:
    req = urllib.request.Request(f"http://127.0.0.1:{port}{route}", data=json.dumps(payload).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=120) as r:
        return json.loads(r.read())


def _wait(port: int, proc, timeout: float = 180.0) -> None:
    t0 = time.monotonic()
    while time.monotonic() - t0 < timeout:
        if proc.poll() is not None:
            raise RuntimeError(f"server exited with {proc.returncode}")
        try:
            with urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=2):
                return
        except OSError:
            time.sleep(0.5)
    raise TimeoutError("server did not come up")


@pytest.mark.integration
def test_tp2_server_matches_single_process(tmp_path):
    from wavelet_b200.configs.config import RLConfig
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.transport.policy import PolicyExporter

    import torch

    env = {**os.environ, "WAVELET_FORCE_CPU": "1", "CUDA_VISIBLE_DEVICES": ""}
    p1, p2 = _free(), _free()
    one = subprocess.Popen([sys.executable, "-m", "wavelet_b200", "inference-server", "@", str(_cfg(tmp_path, "one", p1, 1))],
                           cwd=ROOT, env=env, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, start_new_session=True)
    two = subprocess.Popen([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                            "--master-addr=127.0.0.1", f"--master-port={_free()}", "-m", "wavelet_b200",
                            "inference-server", "@", str(_cfg(tmp_path, "two", p2, 2))],
                           cwd=ROOT, env=env, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, start_new_session=True)
    try:
        _wait(p1, one)
        _wait(p2, two)
        # both start from the same exported policy (the trainer's weights)
        trainer = build_model(PRESETS["tiny"], "cpu", torch.float32, seed=11)
        cfg = RLConfig.model_validate({"output_dir": str(tmp_path / "run")})
        d = PolicyExporter(tmp_path / "run", cfg.policy_transfer).export(trainer, 1)
        for port in (p1, p2):
            assert _post(port, "/load_policy", {"policy_dir": str(d), "step": 1})["policy_step"] == 1
        body = {"prompt_token_ids": [[5, 9, 13, 2, 7], [3, 3, 8]], "max_tokens": 8, "temperature": 0.0}
        a, b = _post(p1, "/v1/completions", body), _post(p2, "/v1/completions", body)
        ta = [c["token_ids"] for c in a["choices"]]
        tb = [c["token_ids"] for c in b["choices"]]
        assert ta == tb and all(len(t) == 8 for t in ta)
        assert b["policy_step"] == 1
    finally:
        for p in (one, two):
            try:
                os.killpg(p.pid, 15)
            except ProcessLookupError:
                pass
            p.wait(timeout=60)
