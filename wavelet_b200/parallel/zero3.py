"""ZeRO-3 parameter sharding: bf16 weights sharded over the data-parallel
group and gathered one unit at a time.

The reference wraps every decoder block in FSDP2 with
``reshard_after_forward`` (trainer/model.py:1136-1195): a block's parameters
are all-gathered before its forward, freed after it, gathered again for its
backward, and its gradients are reduce-scattered as soon as its backward
ends.  Here the model's flat store keeps its full layout but each rank holds
only its contiguous shard (``models.params.ShardedFlatParams``); the units
are the decoder layers plus the "edges" (embedding, final norm, LM head):

* forward: the edges are gathered when ``hidden`` starts; layer ``i`` is
  gathered into one of two staging slots while layer ``i - 1`` computes
  (asynchronous collectives, waited on just before use);
* backward (reverse order): layer ``i`` is gathered again (the last layer is
  still staged from the forward), its gradients accumulate in a zeroed fp32
  staging slot, and are reduced to the ranks that own them (asynchronously;
  the owner adds its part into its gradient shard when the slot is reused);
  the edge gradients are reduced when the embedding's backward ends.

A range of the flat layout is owned by one or two ranks (shards are
contiguous), so the gather is one broadcast from each owner and the gradient
reduction one reduce to each owner: every rank still moves each unit's
bytes once per direction, as in an all-gather / reduce-scatter.  With one
rank the gathers are local copies.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..models.params import ShardedFlatParams


@dataclass
class _Unit:
    names: list[str]
    ranges: list[tuple[int, int, int]] = field(default_factory=list)  # (lo, hi, offset in the staging buffer)
    size: int = 0
    layer: int | None = None


class ParamGatherer:
    def __init__(self, model, group=None, prefetch: bool = True):
        flat = model.flat
        if not isinstance(flat, ShardedFlatParams):
            raise TypeError("ZeRO-3 needs a model built with shard_params=True")
        self.model = model
        self.flat = flat
        self.group = group
        self.world, self.rank = flat.dp_world, flat.dp_rank
        self.prefetch = prefetch
        # asynchronous collectives overlap a gather / reduction with the
        # neighbouring layer's kernels on NCCL; gloo (CPU) runs them in order
        self.async_ok = False
        if self.world > 1:
            self.ranks = [dist.get_global_rank(group, r) if group is not None else r for r in range(self.world)]
            self.async_ok = dist.get_backend(group) == "nccl"
        L = len(model.layers)
        by_layer: list[list[str]] = [[] for _ in range(L)]
        edge: list[str] = []
        for s in flat.specs:
            head, _, _ = s.name.partition(".")
            if head.startswith("l") and head[1:].isdigit() and "." in s.name:
                by_layer[int(head[1:])].append(s.name)
            else:
                edge.append(s.name)
        self.layers = [self._unit(n, i) for i, n in enumerate(by_layer)]
        self.edge = self._unit(edge, None)
        dev, dt = flat.device, flat.compute_dtype
        big = max(u.size for u in self.layers)
        self.wslots = [torch.empty(big, device=dev, dtype=dt) for _ in range(2)]
        self.gslots = [torch.empty(big, device=dev, dtype=torch.float32) for _ in range(2)] if flat.grad is not None else None
        self.wedge = torch.empty(self.edge.size, device=dev, dtype=dt)
        self.gedge = torch.empty(self.edge.size, device=dev, dtype=torch.float32) if flat.grad is not None else None
        self.holds = [None, None]  # layer whose weights each slot holds (valid until the next optimizer step)
        self.pending_w: dict[int, list] = {}  # slot -> works of an in-flight gather
        self.pending_g: dict[int, tuple[list, list]] = {}  # grad slot -> (works, [(staging, local) slices])
        flat.gatherer = self
        model.zero3 = self
        for i, layer in enumerate(model.layers):
            layer.zero3 = self

    def _unit(self, names: list[str], layer: int | None) -> _Unit:
        u = _Unit(names, layer=layer)
        spans = sorted(self.flat.offsets[n] for n in names)
        for off, n in spans:  # merge adjacent parameters into ranges
            if u.ranges and off <= u.ranges[-1][1] + 64:
                lo, hi, b = u.ranges[-1]
                u.ranges[-1] = (lo, max(hi, off + n), b)
            else:
                u.ranges.append((off, off + n, 0))
        b = 0
        out = []
        for lo, hi, _ in u.ranges:
            out.append((lo, hi, b))
            b += hi - lo
        u.ranges, u.size = out, b
        return u

    def _owners(self, lo: int, hi: int):
        S = self.flat.shard_numel
        for r in range(lo // S, min(self.world, (hi - 1) // S + 1)):
            a, b = max(lo, r * S), min(hi, (r + 1) * S)
            if a < b:
                yield r, a, b

    # ------------------------------------------------------------- weights
    def _gather(self, u: _Unit, buf: torch.Tensor, async_op: bool) -> list:
        async_op = async_op and self.async_ok
        works = []
        flat = self.flat
        for lo, hi, b0 in u.ranges:
            for r, a, b in self._owners(lo, hi):
                dst = buf[b0 + a - lo: b0 + b - lo]
                if r == self.rank:
                    dst.copy_(flat.compute[a - flat.lo: b - flat.lo])
                if self.world > 1:
                    w = dist.broadcast(dst, src=self.ranks[r], group=self.group, async_op=async_op)
                    if async_op:
                        works.append(w)
        return works

    def _bind(self, u: _Unit, buf: torch.Tensor, grads: torch.Tensor | None) -> None:
        flat = self.flat
        layer = self.model.layers[u.layer] if u.layer is not None else None
        pre = f"l{u.layer}." if u.layer is not None else ""
        for n in u.names:
            off, k = flat.offsets[n]
            shape = next(s.shape for s in flat.specs if s.name == n)
            b0 = next(b0 + off - lo for lo, hi, b0 in u.ranges if lo <= off < hi)
            flat._staged[n] = buf[b0:b0 + k].view(shape)
            if layer is not None:
                layer.P[n[len(pre):]] = flat._staged[n]
            if grads is not None:
                flat._gstaged[n] = grads[b0:b0 + k].view(shape)
                if layer is not None:
                    layer.G[n[len(pre):]] = flat._gstaged[n]

    def _wait_slot(self, slot: int) -> None:
        for w in self.pending_w.pop(slot, []):
            w.wait()

    def _fetch(self, i: int, async_op: bool) -> None:
        slot = i % 2
        self._wait_slot(slot)
        works = self._gather(self.layers[i], self.wslots[slot], async_op)
        self.holds[slot] = i
        if works:
            self.pending_w[slot] = works

    def _stage(self, i: int, grads: bool, nxt: int | None) -> None:
        slot = i % 2
        if self.holds[slot] != i:
            self._fetch(i, async_op=False)
        self._wait_slot(slot)
        g = None
        if grads and self.gslots is not None:
            self._finish_reduce(slot)
            g = self.gslots[slot]
            g.zero_()
        self._bind(self.layers[i], self.wslots[slot], g)
        if self.prefetch and nxt is not None and 0 <= nxt < len(self.layers) and self.holds[nxt % 2] != nxt:
            self._fetch(nxt, async_op=True)

    # ------------------------------------------------------------- hooks
    def begin_forward(self) -> None:
        """Start of a forward pass: fresh weights (after an optimizer step the
        staged copies are stale), the edges gathered, their gradients zeroed."""
        for s in (0, 1):
            self._wait_slot(s)
        self.holds = [None, None]
        self._gather(self.edge, self.wedge, async_op=False)
        if self.gedge is not None:
            self._finish_all_reduces()
            self.gedge.zero_()
        self._bind(self.edge, self.wedge, self.gedge)

    def stage_forward(self, i: int) -> None:
        self._stage(i, grads=False, nxt=i + 1)

    def stage_backward(self, i: int) -> None:
        self._stage(i, grads=True, nxt=i - 1)

    def end_backward_layer(self, i: int) -> None:
        """Layer ``i``'s gradients are complete: reduce them to their owners."""
        if self.gslots is None:
            return
        slot = i % 2
        self.pending_g[slot] = self._reduce(self.layers[i], self.gslots[slot], async_op=True)

    def finish_backward(self) -> None:
        """End of a backward pass: every layer reduction lands in the
        gradient shards, then the edges' gradients are reduced."""
        if self.gedge is None:
            return
        self._finish_all_reduces()
        works, adds = self._reduce(self.edge, self.gedge, async_op=False)
        self._apply_adds(adds)

    # ------------------------------------------------------------- gradients
    def _reduce(self, u: _Unit, g: torch.Tensor, async_op: bool):
        async_op = async_op and self.async_ok
        works, adds = [], []
        flat = self.flat
        for lo, hi, b0 in u.ranges:
            for r, a, b in self._owners(lo, hi):
                src = g[b0 + a - lo: b0 + b - lo]
                if self.world > 1:
                    w = dist.reduce(src, dst=self.ranks[r], op=dist.ReduceOp.SUM, group=self.group,
                                    async_op=async_op)
                    if async_op:
                        works.append(w)
                if r == self.rank:
                    adds.append((src, slice(a - flat.lo, b - flat.lo)))
        return works, adds

    def _apply_adds(self, adds) -> None:
        for src, sl in adds:
            self.flat.grad[sl].add_(src)

    def _finish_reduce(self, slot: int) -> None:
        p = self.pending_g.pop(slot, None)
        if p is None:
            return
        works, adds = p
        for w in works:
            w.wait()
        self._apply_adds(adds)

    def _finish_all_reduces(self) -> None:
        for s in list(self.pending_g):
            self._finish_reduce(s)

    # ------------------------------------------------------------- full state
    @torch.no_grad()
    def gather_into(self, dst_flat) -> None:
        """Collective: every rank writes the full weights into ``dst_flat``
        (a replicated store of the same layout, e.g. a generator replica):
        one broadcast per owner segment straight into the destination."""
        flat = self.flat
        dst = dst_flat.compute
        if dst_flat.offsets != flat.offsets:
            raise ValueError("the destination store has another layout")
        for u in [self.edge] + self.layers:
            for lo, hi, _ in u.ranges:
                for r, a, b in self._owners(lo, hi):
                    out = dst[a:b]
                    if r == self.rank:
                        out.copy_(flat.compute[a - flat.lo: b - flat.lo])
                    if self.world > 1:
                        dist.broadcast(out, src=self.ranks[r], group=self.group)

    @torch.no_grad()
    def full_state(self, keep) -> dict[str, torch.Tensor] | None:
        """Collective: every parameter's full tensor passed through ``keep(name,
        tensor)`` on data-parallel rank 0 (a host copy for a checkpoint); the
        other ranks take part in the gathers and get None."""
        out = {} if self.rank == 0 else None
        for u, buf in [(self.edge, self.wedge)] + [(u, self.wslots[0]) for u in self.layers]:
            self._wait_slot(0)
            self._gather(u, buf, async_op=False)
            if out is not None:
                for n in u.names:
                    off, k = self.flat.offsets[n]
                    shape = next(s.shape for s in self.flat.specs if s.name == n)
                    b0 = next(b0 + off - lo for lo, hi, b0 in u.ranges if lo <= off < hi)
                    out[n] = keep(n, buf[b0:b0 + k].view(shape))
        self.holds = [None, None]
        return out


class ShardedPolicySync:
    """Generator replica of a ZeRO-3 trainer: a full bf16 store of the same
    layout refreshed from the shards after each optimizer step (every rank
    takes part; the reference's rollout engine gets FSDP-gathered weights the
    same way)."""

    def __init__(self, trainer_model, gen_model):
        self.t = trainer_model
        self.g = gen_model
        if trainer_model.zero3 is None:
            raise ValueError("the trainer model has no ParamGatherer")

    def refresh(self) -> None:
        self.t.zero3.gather_into(self.g.flat)
