"""Ownership partition of a container across GPUs (decode needs no communication).

The container's chunk sequence (tensors in container order, each cut into its
bf16_exp_chunked_v1 chunks) is cut into ``world`` contiguous spans of equal
value count.  A rank owns a few whole tensors plus at most two chunk ranges of
the tensors at its span ends, so rank loads differ by at most one chunk; every
chunk has exactly one owner.  A rank decodes its share from its own HBM
(``DeviceLoader(image, owned=...)`` or plans with ``chunk_begin/chunk_count``);
``bigsmall_b200.replicate`` then materialises the whole model on every rank if
wanted.  The reference has no multi-GPU path (it decodes on the host, one
process); this is the partition a multi-GPU load of its containers uses.
"""
from __future__ import annotations

import math
from typing import Iterable, List, Sequence, Tuple

Owned = List[Tuple[str, int, int]]   # (name, chunk_begin, chunk_count); (name, 0, 0) = whole tensor


def _count(shape_or_n) -> int:
    if isinstance(shape_or_n, int):
        return shape_or_n
    return math.prod(shape_or_n)


def partition(tensors: Iterable[Sequence], world: int, chunk_elems: int) -> Tuple[List[Owned], List[int]]:
    """``tensors``: (name, shape or value count[, ...]) in container order, all
    chunked by ``chunk_elems``.  Returns (owned[rank], values decoded per rank)."""
    return partition_chunks([(t[0], _count(t[1]), chunk_elems) for t in tensors], world)


def partition_chunks(tensors: Iterable[Tuple[str, int, int]], world: int) -> Tuple[List[Owned], List[int]]:
    """As ``partition`` with a chunk size per tensor: (name, n_values, chunk_elems);
    a tensor that cannot be split passes chunk_elems = n (or 0) and is owned whole."""
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    items = []
    for name, n, ce in tensors:
        ce = int(ce) if ce else max(int(n), 1)
        items.append((name, n, ce, max(1, -(-n // ce))))   # an empty tensor is still owned once
    total = sum(n for _, n, _, _ in items)
    owned: List[Owned] = [[] for _ in range(world)]
    load = [0] * world
    r, acc = 0, 0
    for name, n, ce, nc in items:
        c = 0
        while c < nc:
            target = total * (r + 1) / world
            take = nc - c                      # the last rank takes the rest
            if r < world - 1:
                room = target - acc
                fit = max(1, int(round(room / ce))) if room > 0 else 0
                take = min(take, fit) if fit else 0
            if take == 0:
                r += 1
                continue
            e = min(n, (c + take) * ce) - c * ce
            owned[r].append((name, c, take) if (c, take) != (0, nc) else (name, 0, 0))
            load[r] += e
            acc += e
            c += take
            if r < world - 1 and acc >= target - ce / 2:
                r += 1
    return owned, load


def owned_for(header: dict, rank: int, world: int) -> Owned:
    """Rank ``rank``'s share of a container header's tensors (container order):
    bf16_exp_chunked_v1 tensors by chunk spans, every other stored tensor whole
    (``tied_ref`` entries hold no data and go to no rank; a loader resolves
    them to their master)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    items = []
    for t in header["tensors"]:
        codec = t.get("codec")
        if codec == "tied_ref":
            continue
        n = _count(t["shape"])
        items.append((t["name"], n, int(t["extra"]["chunk_elems"]) if codec == "bf16_exp_chunked_v1" else 0))
    return partition_chunks(items, world)[0][rank]
