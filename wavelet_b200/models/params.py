"""Flat parameter storage.

All trainable tensors of a model live in a handful of flat buffers:

* ``compute`` — the compute-dtype copy (bf16 on GPU) that forward/backward
  read; every parameter is a view into it.  It is resident in full on every
  data-parallel rank (a 7B model is 15 GB of a B200's 180 GB).
* ``grad`` — fp32 gradient accumulator in the same layout; kernels accumulate
  weight gradients straight into its views (GEMM fp32-accumulate epilogue).
* ``master``, ``exp_avg``, ``exp_avg_sq`` — fp32 optimizer state, sharded
  across the data-parallel group (rank r owns elements
  [r * shard, (r + 1) * shard)).  After the gradient reduce-scatter each rank
  updates its shard and writes the bf16 shard into ``compute``; an all-gather
  re-replicates ``compute``.

The reference keeps parameters in FSDP1/FSDP2 wrappers with fp32 params and
bf16 compute (trainer/model.py:1048-1195); this is the same numerics with a
layout designed for flat fused kernels and 180 GB of HBM per GPU.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Iterable

import torch

ALIGN = 64  # elements; keeps every view 128-byte aligned in bf16, 256 in fp32


@dataclass
class ParamSpec:
    name: str
    shape: tuple[int, ...]
    init: str = "normal"  # normal | ones | zeros
    # informational: AdamW decays every parameter alike, as the reference's
    # single parameter group does (trainer/optim.py builds one group)
    weight_decay: bool = True
    std: float = 0.02


class FlatParams:
    # ZeRO-3 stores (ShardedFlatParams) hold only this rank's shard of
    # ``compute`` and ``grad``; full parameters exist while a unit is staged
    sharded_compute = False

    def __init__(
        self,
        specs: Iterable[ParamSpec],
        device: torch.device | str,
        compute_dtype: torch.dtype,
        dp_rank: int = 0,
        dp_world: int = 1,
        with_grad: bool = True,
        with_optimizer: bool = True,
        alloc=None,
    ):
        self.specs: list[ParamSpec] = list(specs)
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.dp_rank = dp_rank
        self.dp_world = dp_world
        self.offsets: dict[str, tuple[int, int]] = {}
        off = 0
        for s in self.specs:
            n = math.prod(s.shape)
            self.offsets[s.name] = (off, n)
            off += (n + ALIGN - 1) // ALIGN * ALIGN
        unit = ALIGN * dp_world
        self.numel = (off + unit - 1) // unit * unit
        self.shard_numel = self.numel // dp_world
        # ``alloc(numel, dtype)`` places the replicated buffers in peer-visible
        # memory (parallel.fabric) for the fused collective kernels.
        local = self.shard_numel if self.sharded_compute else self.numel
        if alloc is not None:
            self.compute = alloc(local, compute_dtype)
            self.grad = alloc(local, torch.float32) if with_grad else None
        else:
            self.compute = torch.zeros(local, device=self.device, dtype=compute_dtype)
            self.grad = torch.zeros(local, device=self.device, dtype=torch.float32) if with_grad else None
        self.master = None
        self.exp_avg = None
        self.exp_avg_sq = None
        if with_optimizer:
            self.master = torch.zeros(self.shard_numel, device=self.device, dtype=torch.float32)
            self.exp_avg = torch.zeros_like(self.master)
            self.exp_avg_sq = torch.zeros_like(self.master)
        self._views: dict[str, torch.Tensor] = {}
        self._gviews: dict[str, torch.Tensor] = {}
        # tensor parallelism: the parameters that every TP rank holds whole (and
        # whose gradients are identical on every TP rank) come first, in
        # [0, tp_repl_end); the global gradient norm counts them once
        self.tp_size = 1
        self.tp_repl_end = 0

    def set_tp_replicated(self, names: Iterable[str], tp_size: int) -> None:
        """Marks the leading parameters ``names`` as replicated over ``tp_size``
        tensor-parallel ranks (they must be the first specs of the store)."""
        names = set(names)
        lead = 0
        for s in self.specs:
            if s.name not in names:
                break
            lead += 1
        if lead != len(names):
            raise ValueError("TP-replicated parameters must come first in the flat store")
        end = 0
        for s in self.specs[:lead]:
            off, n = self.offsets[s.name]
            end = max(end, off + (n + ALIGN - 1) // ALIGN * ALIGN)
        self.tp_size = int(tp_size)
        self.tp_repl_end = end

    def shard_repl_split(self) -> int:
        """Number of leading elements of this rank's shard that lie in the
        TP-replicated region."""
        lo = self.dp_rank * self.shard_numel
        return max(0, min(self.tp_repl_end - lo, self.shard_numel))

    # ------------------------------------------------------------- views
    def view(self, name: str) -> torch.Tensor:
        v = self._views.get(name)
        if v is None:
            off, n = self.offsets[name]
            shape = next(s.shape for s in self.specs if s.name == name)
            # views for kernels and I/O never take part in autograd (the CPU
            # reference path slices ``compute`` itself when it needs gradients)
            v = self.compute.detach()[off : off + n].view(shape)
            self._views[name] = v
        return v

    def grad_view(self, name: str) -> torch.Tensor | None:
        if self.grad is None:
            return None
        v = self._gviews.get(name)
        if v is None:
            off, n = self.offsets[name]
            shape = next(s.shape for s in self.specs if s.name == name)
            v = self.grad[off : off + n].view(shape)
            self._gviews[name] = v
        return v

    def names(self) -> list[str]:
        return [s.name for s in self.specs]

    @property
    def shard_slice(self) -> slice:
        """This rank's optimizer shard as a slice of ``compute`` / ``grad``."""
        return slice(self.dp_rank * self.shard_numel, (self.dp_rank + 1) * self.shard_numel)

    @property
    def global_shard_slice(self) -> slice:
        """This rank's optimizer shard in the full flat layout."""
        return slice(self.dp_rank * self.shard_numel, (self.dp_rank + 1) * self.shard_numel)

    # ------------------------------------------------------------- init
    def init_(self, seed: int = 0, std_override: float | None = None, seed_index: dict | None = None,
              row_slices: dict | None = None) -> None:
        """Random init N(0, std) for matrices, ones for norms, zeros for biases.

        Every rank produces identical weights (same generator seed per tensor).
        """
        g = torch.Generator(device=self.device)
        for i, s in enumerate(self.specs):
            v = self.view(s.name)
            if s.init == "ones":
                v.fill_(1.0)
            elif s.init == "zeros":
                v.zero_()
            else:
                g.manual_seed(seed * 1_000_003 + (seed_index[s.name] if seed_index else i))
                std = std_override if std_override is not None else s.std
                # generate in fp32 then cast (bf16 normal_ draws differ by dtype)
                if row_slices and s.name in row_slices:
                    # a shard of a larger tensor (expert / tensor parallelism): draw
                    # the full tensor with its own seed and keep our part, so every
                    # layout of the model holds identical weights.  The entry is
                    # (full shape, lo, hi) for a row range or (full shape, fn) with
                    # fn(full) -> local.
                    ent = row_slices[s.name]
                    tmp = torch.empty(ent[0], device=self.device, dtype=torch.float32)
                    tmp.normal_(0.0, std, generator=g)
                    tmp = ent[1](tmp) if callable(ent[1]) else tmp[ent[1]:ent[2]]
                else:
                    tmp = torch.empty(v.shape, device=self.device, dtype=torch.float32)
                    tmp.normal_(0.0, std, generator=g)
                v.copy_(tmp)
        self.sync_master_from_compute()

    def sync_master_from_compute(self) -> None:
        if self.master is not None:
            self.master.copy_(self.compute[self.shard_slice].float())

    def load_state(self, tensors: dict[str, torch.Tensor], strict: bool = True) -> list[str]:
        missing = []
        for s in self.specs:
            t = tensors.get(s.name)
            if t is None:
                missing.append(s.name)
                continue
            self.view(s.name).copy_(t.reshape(s.shape).to(self.compute_dtype))
        if strict and missing:
            raise KeyError(f"missing parameters: {missing[:8]}{'...' if len(missing) > 8 else ''}")
        self.sync_master_from_compute()
        return missing

    def zero_grad(self) -> None:
        if self.grad is not None:
            self.grad.zero_()

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {s.name: self.view(s.name) for s in self.specs}

    def iter_params(self, fn: Callable[[str, torch.Tensor], None]) -> None:
        for s in self.specs:
            fn(s.name, self.view(s.name))


class ShardedFlatParams(FlatParams):
    """ZeRO-3 flat store: the full layout (offsets) of ``FlatParams``, but each
    data-parallel rank keeps only its shard [r * shard, (r + 1) * shard) of
    the bf16 ``compute`` buffer and of the fp32 ``grad`` buffer (the reduced
    gradients of the elements it owns), next to the fp32 optimizer shard.
    A parameter's full tensor exists only while its unit (a decoder layer, or
    the embedding / final norm / head edges) is staged by a
    ``parallel.zero3.ParamGatherer``: ``view`` / ``grad_view`` then return
    views of the staging buffers (the reference's FSDP2 with
    reshard_after_forward, trainer/model.py:1136-1195)."""

    sharded_compute = True

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.lo = self.dp_rank * self.shard_numel
        self.hi = self.lo + self.shard_numel
        self._staged: dict[str, torch.Tensor] = {}
        self._gstaged: dict[str, torch.Tensor] = {}
        self.gatherer = None  # set by ParamGatherer

    @property
    def shard_slice(self) -> slice:
        return slice(0, self.shard_numel)

    def local_range(self, off: int, n: int) -> tuple[int, int, int, int] | None:
        """(lo, hi) of [off, off + n) held here, in local and in tensor
        coordinates: (local_lo, local_hi, tensor_lo, tensor_hi)."""
        a, b = max(off, self.lo), min(off + n, self.hi)
        if a >= b:
            return None
        return a - self.lo, b - self.lo, a - off, b - off

    def view(self, name: str) -> torch.Tensor:
        v = self._staged.get(name)
        if v is None:
            raise RuntimeError(f"{name} is sharded (ZeRO-3): its unit is not gathered")
        return v

    def grad_view(self, name: str) -> torch.Tensor | None:
        if self.grad is None:
            return None
        v = self._gstaged.get(name)
        if v is None:
            raise RuntimeError(f"the gradient of {name} is sharded (ZeRO-3): its unit is not staged for backward")
        return v

    def init_(self, seed: int = 0, std_override: float | None = None, seed_index: dict | None = None,
              row_slices: dict | None = None) -> None:
        """The same weights as ``FlatParams.init_`` (one generator seed per
        tensor), of which this rank keeps the part in its shard."""
        if row_slices:
            raise NotImplementedError("sharded parameters do not combine with tensor or expert parallelism")
        g = torch.Generator(device=self.device)
        for i, s in enumerate(self.specs):
            off, n = self.offsets[s.name]
            r = self.local_range(off, n)
            if r is None:
                continue
            ll, lh, tl, th = r
            dst = self.compute[ll:lh]
            if s.init == "ones":
                dst.fill_(1.0)
            elif s.init == "zeros":
                dst.zero_()
            else:
                g.manual_seed(seed * 1_000_003 + (seed_index[s.name] if seed_index else i))
                std = std_override if std_override is not None else s.std
                tmp = torch.empty(n, device=self.device, dtype=torch.float32)
                tmp.normal_(0.0, std, generator=g)
                dst.copy_(tmp[tl:th])
                del tmp
        self.sync_master_from_compute()

    def load_state(self, tensors: dict[str, torch.Tensor], strict: bool = True) -> list[str]:
        missing = []
        for s in self.specs:
            t = tensors.get(s.name)
            if t is None:
                missing.append(s.name)
                continue
            off, n = self.offsets[s.name]
            r = self.local_range(off, n)
            if r is not None:
                ll, lh, tl, th = r
                self.compute[ll:lh].copy_(t.reshape(-1)[tl:th].to(self.compute_dtype))
        if strict and missing:
            raise KeyError(f"missing parameters: {missing[:8]}{'...' if len(missing) > 8 else ''}")
        self.sync_master_from_compute()
        return missing

    def state_dict(self) -> dict[str, torch.Tensor]:
        raise RuntimeError("a ZeRO-3 store has no full tensors; gather them (ParamGatherer.full_state)")

    def iter_params(self, fn: Callable[[str, torch.Tensor], None]) -> None:
        raise RuntimeError("a ZeRO-3 store has no full tensors; gather them (ParamGatherer.full_state)")
