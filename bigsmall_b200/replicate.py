"""Materialise a fully replicated model after an ownership-partitioned decode.

Decode needs no communication: each rank decodes its own contiguous span of
the container's values (tensors in name order).  When every GPU must hold the
whole model, each rank's span is broadcast from its owner over NCCL (NVLink /
NVSwitch on one box) into the same offsets of every rank's flat buffer.  The
spans differ in length by up to one chunk, so this is a sequence of
per-owner broadcasts rather than an equal-split all-gather; each broadcast
already drives every link.  Reported separately from the decode throughput.
"""
from __future__ import annotations

from typing import Sequence

import torch


def replicate_spans(flat: torch.Tensor, spans: Sequence[tuple], group=None) -> None:
    """``flat``: the same-shaped 1-D buffer on every rank; ``spans[r] = (lo, hi)``
    is rank r's decoded range.  After the call every rank holds all spans."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if len(spans) != world:
        raise ValueError(f"need one span per rank ({world}), got {len(spans)}")
    b = flat.view(torch.uint8)          # bytes: every backend carries uint8
    es = flat.element_size()
    for r, (lo, hi) in enumerate(spans):
        if hi > lo:
            dist.broadcast(b[lo * es:hi * es], src=dist.get_global_rank(group, r) if group is not None else r,
                           group=group)


def span_checksums(flat: torch.Tensor, spans: Sequence[tuple]) -> torch.Tensor:
    """Per-span int64 sums of the 16-bit words (a size-independent replica check)."""
    w = flat.view(torch.int16)
    return torch.stack([w[lo:hi].to(torch.int64).sum() if hi > lo else torch.zeros((), dtype=torch.int64,
                                                                                    device=flat.device)
                        for lo, hi in spans])
