"""Replicated materialisation after a partitioned decode (bigsmall_b200/
replicate.py), as world-size-2 gloo ranks on CPU: each rank fills only its
own span; afterwards both hold every span, and the per-span checksums agree."""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from bigsmall_b200.replicate import replicate_spans, span_checksums
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 100_003
        spans = [(0, 40_000), (40_000, n)] if world == 2 else None
        full = (torch.arange(n, dtype=torch.int32) * 7 + 3).to(torch.int16)
        flat = torch.zeros(n, dtype=torch.int16)
        lo, hi = spans[rank]
        flat[lo:hi] = full[lo:hi]
        replicate_spans(flat, spans)
        ok = bool(torch.equal(flat, full))
        sums = span_checksums(flat, spans)
        gathered = [torch.zeros_like(sums) for _ in range(world)]
        dist.all_gather(gathered, sums)
        q.put((rank, ok, all(torch.equal(g, gathered[0]) for g in gathered)))
    finally:
        dist.destroy_process_group()


def test_replicate_spans_gloo_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(r for r, _, _ in res) == [0, 1]
    assert all(ok and same for _, ok, same in res), res
