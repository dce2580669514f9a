"""Collation of processor-produced multimodal fields (reference
data/multimodal.py).

A sample may carry ``mm_kwargs``: tensors an HF processor produced next to
``input_ids`` (pixel / video patches, grid shapes, image sizes, per-token
modality ids).  For a batch, every field present in any sample must be present
in all of them; vision tensors are concatenated along their first dimension
(patches of all images in batch order, as vision towers consume them), and
``mm_token_type_ids`` (one id per input token) is right-padded with zeros to
``max_len`` and stacked.  Unknown field names are rejected so that a processor
change cannot silently drop inputs.  ``pack_multimodal_row`` does the same for
one packed row of documents (vision tensors concatenated in document order,
the number of images of every document alongside), which the vision-language
models of ``models.hf_generic`` consume.
"""

from __future__ import annotations

from typing import Any

import torch

VISION_FIELDS = frozenset({"pixel_values", "pixel_values_videos", "image_grid_thw", "video_grid_thw", "image_sizes",
                           "video_sizes", "second_per_grid_ts"})
TOKEN_FIELDS = frozenset({"mm_token_type_ids"})
PROCESSOR_FIELDS = VISION_FIELDS | TOKEN_FIELDS


def collate_multimodal_fields(samples: list[dict[str, Any]], max_len: int) -> dict[str, torch.Tensor]:
    per = [s.get("mm_kwargs") or {} for s in samples]
    names = set().union(*per) if per else set()
    bad = sorted(names - PROCESSOR_FIELDS)
    if bad:
        raise ValueError(f"Unsupported processor fields: {bad}")
    out: dict[str, torch.Tensor] = {}
    for name in sorted(names):
        if any(name not in kw or kw[name] is None for kw in per):
            raise ValueError(f"All samples in a batch must provide multimodal field {name!r}")
        ts = [torch.as_tensor(kw[name]) for kw in per]
        if name in TOKEN_FIELDS:
            for t, s in zip(ts, samples):
                if t.dim() != 1 or t.numel() != len(s["input_ids"]):
                    raise ValueError(f"{name} must have one entry per input token")
                if t.numel() > max_len:
                    raise ValueError(f"{name} is longer than max_len={max_len}")
            out[name] = torch.stack([torch.nn.functional.pad(t, (0, max_len - t.numel())) for t in ts])
        else:
            try:
                out[name] = torch.cat(ts, 0)
            except RuntimeError as e:
                raise ValueError(f"Multimodal field {name!r} has incompatible shapes") from e
    return out


def as_mm_tensors(kw: dict[str, Any] | None) -> dict[str, torch.Tensor] | None:
    """Processor fields of one sample as tensors (JSON rows carry lists)."""
    if not kw:
        return None
    bad = sorted(set(kw) - PROCESSOR_FIELDS)
    if bad:
        raise ValueError(f"Unsupported processor fields: {bad}")
    out = {}
    for k, v in kw.items():
        t = torch.as_tensor(v)
        out[k] = t.long() if k.endswith(("_thw", "_sizes")) or k in TOKEN_FIELDS else t.float() if t.is_floating_point() else t
    return out


def pack_multimodal_row(per_doc: list[dict[str, torch.Tensor] | None]) -> dict[str, Any] | None:
    """The processor fields of a packed row of documents: vision tensors
    concatenated along their first dimension in document order,
    ``doc_images`` = images (grid rows) per document."""
    if not any(per_doc):
        return None
    names = sorted(set().union(*[set(d) for d in per_doc if d]))
    out: dict[str, Any] = {}
    for n in names:
        if n in TOKEN_FIELDS:
            raise ValueError(f"{n} is not supported in packed rows")
        parts = [d[n] for d in per_doc if d and n in d]
        out[n] = torch.cat(parts, 0)
    grid = "image_grid_thw"
    out["doc_images"] = [int(d[grid].shape[0]) if d and grid in d else 0 for d in per_doc]
    return out
