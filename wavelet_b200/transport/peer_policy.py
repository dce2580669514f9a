"""Device policy transfer for the split placement (``policy_transfer.type:
nccl`` with the trainer and the generator in separate processes).

The reference moves a policy with a layer-by-layer NCCL broadcast from
trainer rank 0 into paused vLLM workers, after a ready handshake
(transport/policy.py:355-560, 782-930).  Here, when the generator GPUs sit in
the trainer's NVLink node, the transfer is a push over peer memory:

* every generator process (``PeerPolicyReceiver``) allocates ``slots``
  receive buffers in its own layout and a small control pad, exports CUDA IPC
  handles for them and describes them in ``<policy_dir>/peer/receiver-<i>.json``;
* every trainer rank (``PeerPolicySender``) opens those handles and, with one
  ``policy_push`` launch per source buffer, stores the part of the weights it
  holds into slot ``step % slots`` of every generator: tensor-parallel row /
  column blocks and expert-parallel expert blocks land at their place in the
  full tensors, cast to the generator's dtype on the way.  Ranks that hold the
  same data split the work between them;
* pad word ``k`` holds the epoch (step + 1) of slot ``k``; trainer rank 0
  zeroes it before the slot is rewritten and release-stores the new epoch
  after every rank's stores are done.  The trainer never waits for a
  generator;
* a generator loads a step by copying the newest complete slot into its
  weights between generation batches and re-reading the epoch afterwards: an
  epoch that changed while it copied (the trainer overwrote that slot) makes
  it copy again (a sequence lock).

Across nodes the NCCL fallback (``PolicyBroadcastGroup``) broadcasts the flat
bf16 buffer from trainer rank 0 over a dedicated process group built from a
TCP store (``nccl_host`` / ``nccl_port``), with the reference's ready marker
handshake; it needs identical flat layouts (no tensor or expert parallelism
on the trainer).
"""

from __future__ import annotations

import json
import os
import socket
import time
from dataclasses import dataclass
from datetime import timedelta
from pathlib import Path
from typing import Any, Callable

import torch

PROTOCOL = "peer_v1"
FLAT_PROTOCOL = "flat_v1"
PEER_DIR = "peer"
READY_PREFIX = "ready-"
PAD_WORDS = 256


class PeerUnavailable(RuntimeError):
    """The peer path cannot be used (other host, missing receivers)."""


# ---------------------------------------------------------------- segments
# A segment is one 2-D block (rows x row_len elements) copied from a source
# buffer to a destination buffer: (src_off, dst_off, rows, row_len,
# src_stride, dst_stride), offsets and strides in elements.

def _contig(src_off: int, dst_off: int, n: int) -> tuple:
    return (src_off, dst_off, 1, n, n, n)


def tp_blocks(suffix: str, cfg, tp: int, r: int, src_off: int, dst_off: int) -> list[tuple]:
    """Blocks that place tensor-parallel rank ``r``'s part of a split
    parameter into the full tensor (the inverse of the Megatron slicers: qkv by
    heads and gate/up by rows are row blocks, o and down are column blocks)."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    q, kv = cfg.q_dim, cfg.kv_dim
    ql, kvl, il = q // tp, kv // tp, I // tp
    if suffix in ("qkv_w", "qkv_b"):
        w = H if suffix == "qkv_w" else 1
        runs = [(0, r * ql, ql), (ql, q + r * kvl, kvl), (ql + kvl, q + kv + r * kvl, kvl)]
        return [_contig(src_off + a * w, dst_off + b * w, n * w) for a, b, n in runs]
    if suffix == "gu_w":
        return [_contig(src_off, dst_off + r * il * H, il * H),
                _contig(src_off + il * H, dst_off + (I + r * il) * H, il * H)]
    if suffix == "o_w":
        return [(src_off, dst_off + r * ql, H, ql, ql, q)]
    if suffix == "down_w":
        return [(src_off, dst_off + r * il, H, il, il, I)]
    raise KeyError(f"no tensor-parallel layout for {suffix}")


def _share(segs: list[tuple], index: int, count: int) -> list[tuple]:
    """This replica's part of work that ``count`` identical replicas split:
    segments sorted by size, each to the least loaded replica (deterministic,
    so every replica computes the same assignment)."""
    if count <= 1:
        return list(segs)
    load = [0] * count
    mine = []
    for i in sorted(range(len(segs)), key=lambda i: (-segs[i][2] * segs[i][3], i)):
        j = min(range(count), key=lambda j: (load[j], j))
        load[j] += segs[i][2] * segs[i][3]
        if j == index:
            mine.append(segs[i])
    return mine


def push_segments(model, gen_offsets: dict[str, tuple[int, int]], rank: int = 0, world: int = 1
                  ) -> dict[str, list[tuple]]:
    """Segments of this trainer rank, per source buffer (``"flat"``: the
    compute store; ``"expert"``: the expert store under expert parallelism),
    that write the generator layout ``gen_offsets`` (name -> (offset, numel)
    of the full tensors)."""
    from ..models.qwen import tp_slicers

    if getattr(model, "lora", None) is not None or getattr(model, "quant", None):
        raise NotImplementedError("device policy transfer moves full-model weights; LoRA / NF4 trainers use the "
                                  "filesystem transfer (the adapter is small)")
    cfg = model.cfg
    if getattr(model.flat, "sharded_compute", False):
        # ZeRO-3: each rank pushes exactly the elements of its shard
        flat = model.flat
        segs = []
        for name, (goff, gn) in gen_offsets.items():
            if name not in flat.offsets:
                raise KeyError(f"generator parameter {name} is not held by the trainer")
            off, n = flat.offsets[name]
            if n != gn:
                raise ValueError(f"{name}: trainer has {n} elements, the generator {gn}")
            r = flat.local_range(off, n)
            if r is not None:
                ll, lh, tl, th = r
                segs.append(_contig(ll, goff + tl, lh - ll))
        return {"flat": segs} if segs else {}
    tp, tr = getattr(model, "tp_size", 1), getattr(model, "tp_rank", 0)
    split = set(tp_slicers(cfg, tp, tr)) if tp > 1 else set()
    ef = getattr(model, "expert_flat", None)
    ep = getattr(model, "ep_size", 1)
    full = {"flat": [], "expert": []}
    shared = {"flat": [], "split": [], "expert": []}
    for name, (goff, gn) in gen_offsets.items():
        suffix = name.split(".", 1)[-1]
        if ef is not None and name in ef.offsets:
            off, n = ef.offsets[name]
            if n * ep != gn:
                raise ValueError(f"{name}: {ep} expert shards of {n} do not make {gn}")
            shared["expert"].append(_contig(off, goff + model.ep_rank * n, n))
        elif name in model.flat.offsets:
            off, n = model.flat.offsets[name]
            if suffix in split:
                if n * tp != gn:
                    raise ValueError(f"{name}: {tp} tensor-parallel parts of {n} do not make {gn}")
                shared["split"].extend(tp_blocks(suffix, cfg, tp, tr, off, goff))
            else:
                if n != gn:
                    raise ValueError(f"{name}: trainer has {n} elements, the generator {gn}")
                shared["flat"].append(_contig(off, goff, n))
        else:
            raise KeyError(f"generator parameter {name} is not held by the trainer")
    full["flat"] = _share(shared["flat"], rank, world) + _share(shared["split"], rank // tp, world // tp)
    if ef is not None:
        full["expert"] = _share(shared["expert"], getattr(model, "ep_dp_rank", 0), max(1, world // ep))
    return {k: v for k, v in full.items() if v}


def apply_segments(src: torch.Tensor, segs: list[tuple], dst: torch.Tensor) -> None:
    """The push with torch views (the CPU path and the test oracle)."""
    for so, do, rows, n, ss, ds in segs:
        d = dst.as_strided((rows, n), (ds, 1), dst.storage_offset() + do)
        d.copy_(src.as_strided((rows, n), (ss, 1), src.storage_offset() + so))


# ---------------------------------------------------------------- memory
class _HostMemory:
    """In-process stand-in for peer memory (CPU tests): buffers are tensors in
    a registry, handles are registry keys."""

    _reg: dict[str, torch.Tensor] = {}

    def alloc(self, numel: int, dtype: torch.dtype, device) -> tuple[torch.Tensor, str, int]:
        t = torch.zeros(numel, dtype=dtype)
        key = f"host:{os.getpid()}:{id(t)}"
        self._reg[key] = t
        return t, key, 0

    def open(self, handle: str, numel: int, dtype: torch.dtype, device) -> tuple[Any, int]:
        if handle not in self._reg:
            raise PeerUnavailable("host buffers are only reachable inside their own process")
        return self._reg[handle], 0

    def close(self, opened: int) -> None:
        pass

    def free(self, owned: int, handle: str = "") -> None:
        self._reg.pop(handle, None)


class _CudaMemory:
    """cudaMalloc buffers with CUDA IPC handles (the peer fabric's allocator)."""

    _local: dict[str, int] = {}  # handles of this process -> pointer (IPC cannot open them here)

    def __init__(self):
        from .. import ops

        self.m = ops.ext()

    def alloc(self, numel: int, dtype: torch.dtype, device) -> tuple[torch.Tensor, str, int]:
        dev = torch.device(device).index
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        p = self.m.fabric_malloc(nbytes, dev)
        t = self.m.from_ptr(p, numel, dtype, dev)
        t.zero_()
        torch.cuda.synchronize(device)
        h = self.m.fabric_export(p).hex()
        self._local[h] = p
        return t, h, p

    def open(self, handle: str, numel: int, dtype: torch.dtype, device) -> tuple[int, int]:
        if handle in self._local:
            return self._local[handle], 0
        q = self.m.fabric_import(bytes.fromhex(handle), torch.device(device).index)
        return q, q

    def close(self, opened: int) -> None:
        if opened:
            self.m.fabric_close(opened)

    def free(self, owned: int, handle: str = "") -> None:
        self._local.pop(handle, None)
        if owned:
            self.m.fabric_free(owned)


def _memory_for(device) -> Any:
    return _CudaMemory() if torch.device(device).type == "cuda" else _HostMemory()


def _atomic_json(path: Path, obj: dict) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    tmp.write_text(json.dumps(obj))
    os.replace(tmp, path)


# ---------------------------------------------------------------- receiver
class PeerPolicyReceiver:
    """Generator side: receive slots + control pad, described for senders."""

    def __init__(self, model, policy_dir: Path, index: int = 0, slots: int = 2):
        if slots not in (1, 2):
            raise ValueError("peer policy slots must be 1 or 2")
        self.model = model
        self.index = index
        self.slots = slots
        self.dir = Path(policy_dir) / PEER_DIR
        flat = model.flat
        self.numel = flat.compute.numel()
        self.dtype = flat.compute.dtype
        dev = flat.compute.device
        self.mem = _memory_for(dev)
        self.bufs, self.handles, self.owned = [], [], []
        for _ in range(slots):
            t, h, p = self.mem.alloc(self.numel, self.dtype, dev)
            self.bufs.append(t)
            self.handles.append(h)
            self.owned.append(p)
        self.pad, self.pad_handle, self.pad_owned = self.mem.alloc(PAD_WORDS, torch.int32, dev)
        self.loaded_epoch = 0
        self.path = self.dir / f"receiver-{index}.json"
        _atomic_json(self.path, {
            "format": PROTOCOL, "index": index, "hostname": socket.gethostname(), "pid": os.getpid(),
            "device": str(dev), "numel": self.numel, "dtype": str(self.dtype).removeprefix("torch."),
            "slots": self.handles, "pad": self.pad_handle,
            "layout": {n: list(v) for n, v in flat.offsets.items()}})

    def epochs(self) -> list[int]:
        return [int(x) for x in self.pad[: self.slots].tolist()]

    def load(self, step: int, timeout_s: float = 600.0, poll_s: float = 0.002) -> int:
        """Copy the newest complete slot whose epoch reaches ``step + 1`` into
        the model's weights; returns the step loaded (>= ``step``)."""
        want = step + 1
        deadline = time.monotonic() + timeout_s
        while True:
            ep = self.epochs()
            k = max(range(self.slots), key=lambda i: ep[i])
            e = ep[k]
            if e >= want:
                self.model.flat.compute.copy_(self.bufs[k])
                if self.model.flat.compute.is_cuda:
                    torch.cuda.synchronize(self.model.flat.compute.device)
                if self.epochs()[k] == e:  # not overwritten while we copied
                    self.loaded_epoch = e
                    return e - 1
                continue
            if time.monotonic() > deadline:
                raise TimeoutError(f"policy step {step} did not arrive in receiver {self.index} within {timeout_s}s "
                                   f"(slot epochs {ep})")
            time.sleep(poll_s)

    def close(self) -> None:
        try:
            self.path.unlink()
        except OSError:
            pass
        if self.model.flat.compute.is_cuda:
            torch.cuda.synchronize(self.model.flat.compute.device)
        for p, h in zip(self.owned, self.handles):
            self.mem.free(p, h)
        self.mem.free(self.pad_owned, self.pad_handle)
        self.bufs = []


def read_receivers(policy_dir: Path) -> list[dict]:
    out = []
    for p in sorted((Path(policy_dir) / PEER_DIR).glob("receiver-*.json")):
        try:
            out.append(json.loads(p.read_text()))
        except (OSError, ValueError):
            continue
    return sorted(out, key=lambda d: d["index"])


# ---------------------------------------------------------------- sender
@dataclass
class _Dest:
    desc: dict
    slots: list[Any]  # pointer (cuda) or tensor (host) per slot
    pad: Any
    opened: list[int]


class PeerPolicySender:
    """Trainer side: one instance per trainer rank (all ranks call ``push``).

    ``barrier`` orders the ranks (a process-group barrier); ``expect`` is the
    number of receivers to wait for (bounded by ``timeout_s``)."""

    def __init__(self, model, policy_dir: Path, *, rank: int = 0, world: int = 1, expect: int = 1,
                 timeout_s: float = 600.0, barrier: Callable[[], None] | None = None):
        self.model = model
        self.rank, self.world = rank, world
        self.barrier = barrier or (lambda: None)
        self.dev = model.flat.compute.device
        self.mem = _memory_for(self.dev)
        deadline = time.monotonic() + timeout_s
        while True:
            descs = read_receivers(policy_dir)
            if len(descs) >= expect:
                break
            if time.monotonic() > deadline:
                raise PeerUnavailable(f"{len(descs)} of {expect} policy receivers announced in {policy_dir}")
            time.sleep(0.05)
        host = socket.gethostname()
        if any(d["hostname"] != host for d in descs):
            raise PeerUnavailable("a policy receiver runs on another host")
        layout = {n: (int(v[0]), int(v[1])) for n, v in descs[0]["layout"].items()}
        if any(d["layout"] != descs[0]["layout"] or d["dtype"] != descs[0]["dtype"] for d in descs):
            raise ValueError("policy receivers disagree on the layout")
        self.slots = min(len(d["slots"]) for d in descs)
        self.dst_numel = int(descs[0]["numel"])
        self.dst_dtype = getattr(torch, descs[0]["dtype"])
        self.segs = push_segments(model, layout, rank, world)
        self.dests: list[_Dest] = []
        for d in descs:
            opened, slots = [], []
            for h in d["slots"][: self.slots]:
                p, o = self.mem.open(h, self.dst_numel, self.dst_dtype, self.dev)
                slots.append(p)
                opened.append(o)
            pad, o = self.mem.open(d["pad"], PAD_WORDS, torch.int32, self.dev)
            opened.append(o)
            self.dests.append(_Dest(d, slots, pad, opened))
        self.bytes = sum(s[2] * s[3] for v in self.segs.values() for s in v) * self.dst_dtype.itemsize
        self.push_seconds = 0.0

    def _sources(self) -> dict[str, torch.Tensor]:
        out = {"flat": self.model.flat.compute}
        if getattr(self.model, "expert_flat", None) is not None:
            out["expert"] = self.model.expert_flat.compute
        return out

    def _signal(self, word: int, value: int) -> None:
        if self.dev.type == "cuda":
            from .. import ops

            m = ops.ext()
            for i in range(0, len(self.dests), 8):
                m.policy_signal([d.pad for d in self.dests[i:i + 8]], word, value)
            torch.cuda.synchronize(self.dev)
        else:
            for d in self.dests:
                d.pad[word] = value

    @torch.no_grad()
    def push(self, step: int) -> dict[str, Any]:
        k, e = step % self.slots, step + 1
        t0 = time.perf_counter()
        if self.rank == 0:
            self._signal(k, 0)  # the slot is about to change: no generator starts copying it
        self.barrier()
        src = self._sources()
        cuda = self.dev.type == "cuda"
        if cuda:
            from .. import ops

            m = ops.ext()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record()
        for name, segs in self.segs.items():
            if cuda:
                table = torch.tensor(segs, dtype=torch.int64).reshape(-1, 6)
                for i in range(0, len(self.dests), 8):
                    group = self.dests[i:i + 8]
                    m.policy_push(src[name], [d.slots[k] for d in group], self.dst_numel,
                                  self.dst_dtype == torch.bfloat16, table)
            else:
                for d in self.dests:
                    apply_segments(src[name], segs, d.slots[k])
        kernel_ms = 0.0
        if cuda:
            ev[1].record()
            torch.cuda.synchronize(self.dev)
            kernel_ms = ev[0].elapsed_time(ev[1])
        self.barrier()
        if self.rank == 0:
            self._signal(k, e)
        self.push_seconds = time.perf_counter() - t0
        return {"protocol": PROTOCOL, "slot": k, "epoch": e, "receivers": len(self.dests),
                "bytes_per_receiver_this_rank": self.bytes, "kernel_ms": kernel_ms,
                "push_seconds": self.push_seconds}

    def close(self) -> None:
        if self.dev.type == "cuda":
            torch.cuda.synchronize(self.dev)
        for d in self.dests:
            for o in d.opened:
                self.mem.close(o)
        self.dests = []


# ---------------------------------------------------------------- NCCL fallback
class PolicyBroadcastGroup:
    """A process group of trainer rank 0 (rank 0) and the generator processes
    (ranks ``rank_offset + i``) built from its own TCP store, independent of
    the trainer's default group (the reference uses vLLM's stateless group
    and PyNccl communicator for this, transport/policy.py:355-385)."""

    def __init__(self, host: str, port: int, rank: int, world: int, device, timeout_s: int = 600,
                 backend: str = "nccl"):
        import torch.distributed as dist

        self.rank, self.world = rank, world
        self.device = torch.device(device)
        to = timedelta(seconds=timeout_s)
        self.store = dist.TCPStore(host, port, world, is_master=rank == 0, timeout=to)
        pre = dist.PrefixStore("wavelet_policy", self.store)
        if backend == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts._timeout = to
            self.pg = dist.ProcessGroupNCCL(pre, rank, world, opts)
        else:
            self.pg = dist.ProcessGroupGloo(pre, rank, world, to)

    def broadcast(self, t: torch.Tensor, src: int = 0) -> None:
        import torch.distributed as dist

        opts = dist.BroadcastOptions()
        opts.rootRank = src
        opts.rootTensor = 0
        self.pg.broadcast([t], opts).wait()

    def close(self) -> None:
        try:
            self.pg.shutdown()
        except Exception:
            pass


def used_numel(flat) -> int:
    """Elements of a flat store that hold parameters (the padding excluded)."""
    return max((off + n for off, n in flat.offsets.values()), default=0)


def wait_ready(step_dir: Path, count: int, timeout_s: float) -> None:
    """Trainer rank 0 waits until ``count`` generators entered the update."""
    deadline = time.monotonic() + timeout_s
    while len(list(Path(step_dir).glob(READY_PREFIX + "*"))) < count:
        if time.monotonic() > deadline:
            raise TimeoutError(f"generators did not enter the policy update of {step_dir} within {timeout_s}s")
        time.sleep(0.05)


def mark_ready(step_dir: Path, index: int) -> None:
    (Path(step_dir) / f"{READY_PREFIX}{index}").touch()
