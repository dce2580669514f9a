"""A tensor-parallel generator replica behind one HTTP server
(``inference.vllm.tensor_parallel_size`` > 1; the reference gets this from
vLLM's tensor parallelism, inference/server.py:693-1036).

The replica runs as ``tensor_parallel_size`` processes (one per GPU, started
with torchrun).  Each builds its Megatron part of the model (heads and FFN
columns; row-parallel outputs summed over the group inside the generator).
Rank 0 serves HTTP; every engine call it makes is first broadcast to the
other ranks over a gloo control group, then every rank runs it, so the TP
collectives inside generation line up.  Results come from rank 0.

Policies arrive through the filesystem: every rank loads its part of the
exported checkpoint (``load_hf_weights`` slices the split parameters).
"""

from __future__ import annotations

import os
import threading
from datetime import timedelta
from typing import Any

import torch
import torch.distributed as dist

# engine methods that run on every rank; everything else is read on rank 0
COLLECTIVE = ("generate_ids", "annotate", "score", "load_policy", "sleep", "wake")
_STOP = "__stop__"


class TPEngineProxy:
    """Rank 0's view of the TP engine: collective methods are announced to
    the other ranks before they run here; attributes read through."""

    def __init__(self, engine, ctrl_group):
        self._engine = engine
        self._ctrl = ctrl_group
        self._lock = threading.Lock()  # one collective call at a time, in the same order on every rank

    def __getattr__(self, name: str):
        attr = getattr(self._engine, name)
        if name not in COLLECTIVE:
            return attr

        def call(*args, **kwargs):
            with self._lock:
                dist.broadcast_object_list([(name, args, kwargs)], src=0, group=self._ctrl)
                return attr(*args, **kwargs)

        return call

    def close(self) -> None:
        with self._lock:
            dist.broadcast_object_list([(_STOP, (), {})], src=0, group=self._ctrl)
        self._engine.close()


def worker_loop(engine, ctrl_group) -> None:
    """Ranks > 0: run every call rank 0 announces, until it stops."""
    while True:
        msg: list[Any] = [None]
        dist.broadcast_object_list(msg, src=0, group=ctrl_group)
        name, args, kwargs = msg[0]
        if name == _STOP:
            break
        getattr(engine, name)(*args, **kwargs)
    engine.close()


def build_tp_engine(cfg):
    """This process's engine of a TP replica (torchrun environment)."""
    from ..data.tokenizer import tokenizer_for
    from ..models.config import resolve_arch
    from ..models.qwen import build_model
    from .policy import NativePolicyInferenceEngine

    tp = cfg.inference.vllm.tensor_parallel_size
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != tp:
        raise ValueError(f"inference.vllm.tensor_parallel_size={tp} needs {tp} processes (torchrun), got {world}")
    if cfg.policy_transfer.type == "nccl":
        raise NotImplementedError("a tensor-parallel generator replica takes its policies from the filesystem "
                                  "(policy_transfer.type: filesystem)")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    use_cuda = torch.cuda.is_available() and os.environ.get("WAVELET_FORCE_CPU") != "1"
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    if not dist.is_initialized():
        dist.init_process_group("nccl" if use_cuda else "gloo", timeout=timedelta(seconds=600),
                                **({"device_id": dev} if use_cuda else {}))
    ctrl = dist.new_group(backend="gloo")
    arch = resolve_arch(cfg.model.name, cfg.model.arch_overrides or None)
    model = build_model(arch, dev, torch.bfloat16 if use_cuda else torch.float32, seed=cfg.seed, with_grad=False,
                        with_optimizer=False, tp=(tp, rank))
    model.tp_group = dist.group.WORLD
    engine = NativePolicyInferenceEngine(cfg, model=model, tokenizer=tokenizer_for(cfg.model))
    engine.setup()
    return engine, ctrl, rank


def run_tp_server(cfg) -> int:
    engine, ctrl, rank = build_tp_engine(cfg)
    if rank != 0:
        worker_loop(engine, ctrl)
        dist.destroy_process_group()
        return 0
    import uvicorn

    from .server import build_app

    proxy = TPEngineProxy(engine, ctrl)
    app = build_app(cfg, engine=proxy)
    try:
        uvicorn.run(app, host=cfg.inference.http.host, port=cfg.inference.http.port, log_level="warning")
    finally:
        proxy.close()
        dist.destroy_process_group()
    return 0
