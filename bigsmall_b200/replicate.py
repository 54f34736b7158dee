"""Materialise a fully replicated model after an ownership-partitioned decode.

Decode needs no communication: each rank decodes its own contiguous span of
the container's values (tensors in name order).  When every GPU must hold the
whole model, every rank sends its span to every other rank and receives
theirs into the same offsets of its flat buffer: one batch of point-to-point
transfers over NCCL (NVLink / NVSwitch on one box), all in flight together so
every GPU's links carry traffic in both directions.  The spans differ in
length by up to one chunk, which an equal-split all-gather would not allow.
Reported separately from the decode throughput.
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
    me = dist.get_rank(group)
    glob = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    lo, hi = spans[me]
    ops = []
    for r in range(world):
        if r == me:
            continue
        if hi > lo:
            ops.append(dist.P2POp(dist.isend, b[lo * es:hi * es], glob(r), group))
        rlo, rhi = spans[r]
        if rhi > rlo:
            ops.append(dist.P2POp(dist.irecv, b[rlo * es:rhi * es], glob(r), group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()


def span_checksums(flat: torch.Tensor, spans: Sequence[tuple]) -> torch.Tensor:
    """Per-span int64 sums of the 16-bit words (a size-independent replica check)."""
    w = flat.view(torch.int16)
    return torch.stack([w[lo:hi].to(torch.int64).sum() if hi > lo else torch.zeros((), dtype=torch.int64,
                                                                                    device=flat.device)
                        for lo, hi in spans])
