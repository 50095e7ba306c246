"""In-place weight updates of a serving model (e.g. from a training loop).

The new weights are built by the ordinary loader into a second model object
of the same architecture and parallel layout, then every weight tensor is
copied into the live model's tensor at the same place, so every buffer the
captured CUDA graphs read keeps its address.  Caches derived from old
weights are dropped (the router's bf16 gate copies) and the caller flushes
the prefix cache, whose KV rows came from the old weights.
"""
from __future__ import annotations

from typing import Iterator, Tuple

import torch

# model attributes that hold weights (everything else is state: KV caches,
# tables, streams, tracer, ...)
WEIGHT_ATTRS = ("layers", "embed", "final_ln", "lm_head", "hc_head", "mtp")
_MTP_ATTRS = ("block", "enorm", "hnorm", "eh_proj")


def _walk(obj, path: str, seen) -> Iterator[Tuple[str, torch.Tensor]]:
    if isinstance(obj, torch.Tensor):
        yield path, obj
        return
    if obj is None or isinstance(obj, (int, float, str, bool)) or id(obj) in seen:
        return
    seen.add(id(obj))
    if isinstance(obj, (list, tuple)):
        for i, v in enumerate(obj):
            yield from _walk(v, f"{path}[{i}]", seen)
    elif isinstance(obj, dict):
        for k in sorted(obj):
            yield from _walk(obj[k], f"{path}[{k!r}]", seen)
    elif type(obj).__name__ == "MTPDraft":
        for a in _MTP_ATTRS:
            yield from _walk(getattr(obj, a), f"{path}.{a}", seen)
    elif type(obj).__name__ in ("DeepseekModel", "DeepseekV4Model"):
        for a in WEIGHT_ATTRS:
            yield from _walk(getattr(obj, a, None), f"{path}.{a}", seen)
    elif hasattr(obj, "__dict__"):
        for k, v in sorted(vars(obj).items()):
            yield from _walk(v, f"{path}.{k}", seen)


def weight_tensors(model):
    """(path, tensor) for every weight tensor of a model, in a fixed order."""
    return list(_walk(model, "model", set()))


def copy_weights(dst_model, src_model) -> int:
    """Copy src_model's weights into dst_model's tensors in place; returns
    the number of bytes copied.  The two must have the same structure."""
    dst, src = weight_tensors(dst_model), weight_tensors(src_model)
    if [p for p, _ in dst] != [p for p, _ in src]:
        raise ValueError("weight update: the new weights have a different structure")
    n = 0
    with torch.no_grad():
        for (p, d), (_, s) in zip(dst, src):
            if d.shape != s.shape or d.dtype != s.dtype:
                raise ValueError(f"weight update: {p} is {tuple(s.shape)} {s.dtype}, "
                                 f"the model holds {tuple(d.shape)} {d.dtype}")
            d.copy_(s)
            n += d.numel() * d.element_size()
            # derived copies kept on a weight (the router's bf16 gate) are
            # refreshed in place: captured decode graphs read their buffers
            hit = getattr(d, "_b200_bf16", None)
            if hit is not None:
                hit[1].copy_(d)
                hit[0] = d._version
    return n
