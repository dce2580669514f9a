"""NVTX ranges for timeline tools (Nsight Systems, ncu ``--nvtx``).

Off by default; ``WAVELET_NVTX=1`` (or ``enable(True)``) turns every
``nvtx.range("...")`` in the framework into a push/pop pair on the CUDA
timeline: decoder layers (forward / backward), the LM-head loss, optimizer
steps, the fused collectives and the generator's decode windows.  Disabled,
a range costs one attribute check.
"""

from __future__ import annotations

import os
from contextlib import contextmanager

_ON = os.environ.get("WAVELET_NVTX", "") not in ("", "0")


def enable(on: bool = True) -> None:
    global _ON
    _ON = bool(on)


def enabled() -> bool:
    return _ON


@contextmanager
def range(name: str):  # noqa: A001 - mirrors torch.cuda.nvtx.range
    if not _ON:
        yield
        return
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
