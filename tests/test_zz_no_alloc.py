"""The allocation-free decode entry point, bs_xc_decode_noalloc.

Some callers of this library cannot allocate device memory at decode time: a
serving engine that has already reserved nearly all of HBM for its own arena
or KV cache (a fresh cudaMalloc can fail there), or a latency-critical path
where cudaMalloc/cudaFree would synchronise the whole device.  For them the
library offers one entry point whose scratch (descriptors, decode tables,
status words) is a static device array instead of plan memory.

These tests call it through the C ABI, two calls in a row -- the second call
runs on the scratch the first one left behind -- and check every output bit
for bit against the plan-based entry point (bs_xc_plan_create /
bs_plan_decode) and against the values that were encoded.  One test checks
the promise itself: after a warm-up call, a further call leaves the device's
free memory unchanged.  The file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402


def _tensor(n, seed, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).to(torch.bfloat16)


def _blob(x, coder, ce):
    raw = x.view(torch.uint8).numpy().tobytes()
    b = O.xc_encode(raw, coder, 12, ce)
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).cuda()


def _cases(seed0, with_values=False):
    """(blob, n_total, chunk_elems, chunk_begin, chunk_count) per tensor, and
    with `with_values` also the encoded values (host bf16) of each tensor."""
    specs = [(300_001, 0, 65536, 0, 0), (4096, 1, 256, 0, 0), (1_000_003, 0, 4096, 10, 50),
             (77, 1, 256, 0, 0), (200_000, 0, 65536, 1, 0), (150_001, 2, 4096, 3, 20), (9_999, 2, 256, 0, 0)]
    out, values = [], []
    for i, (n, coder, ce, c0, cc) in enumerate(specs):
        x = _tensor(n, seed0 + i, scale=0.01 * (i + 1))
        out.append((_blob(x, coder, ce), n, ce, c0, cc))
        values.append(x)
    return (out, values) if with_values else out


def _expected_slice(x, n, ce, c0, cc):
    """The values a chunk range [c0, c0 + cc) decodes to (cc 0: to the end)."""
    nc = -(-n // ce)
    cnt = cc if cc else nc - c0
    return x.view(torch.int16)[c0 * ce:min(n, (c0 + cnt) * ce)]


def _outputs(cases):
    outs = []
    for blob, n, ce, c0, cc in cases:
        nc = -(-n // ce)
        cnt = cc if cc else nc - c0
        m = min(n, (c0 + cnt) * ce) - c0 * ce
        outs.append(torch.full((m,), -1, dtype=torch.int16, device="cuda"))
    return outs


def _noalloc(cases, outs):
    from bigsmall_b200 import _lib
    L = _lib.load()
    arr = (_lib.XcTensor * len(cases))()
    for i, ((blob, n, ce, c0, cc), o) in enumerate(zip(cases, outs)):
        arr[i].d_blob = blob.data_ptr()
        arr[i].blob_bytes = blob.numel()
        arr[i].d_out = o.data_ptr()
        arr[i].n_elems = n
        arr[i].chunk_elems = ce
        arr[i].chunk_begin = c0
        arr[i].chunk_count = cc
        arr[i].coder_mask = 0
    st = (ctypes.c_uint32 * max(1, len(cases)))()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.bs_xc_decode_noalloc(arr, len(cases), stream, st)
    return rc, [int(st[i]) for i in range(len(cases))]


def _with_plan(cases):
    from bigsmall_b200 import gpu
    outs = _outputs(cases)
    with gpu.XcPlan([(b, o, ce, n, c0, cc) for (b, n, ce, c0, cc), o in zip(cases, outs)]) as p:
        p.run()
    return outs


def test_noalloc_matches_plan_entry_point_on_consecutive_calls():
    a, va = _cases(100, with_values=True)
    b, vb = _cases(200, with_values=True)
    b, vb = b[:3], vb[:3]
    for cases, values in ((a, va), (b, vb), (a, va)):   # consecutive calls reuse the shared scratch
        want = _with_plan(cases)
        got = _outputs(cases)
        rc, st = _noalloc(cases, got)
        assert rc == 0 and st == [0] * len(cases), (rc, st)
        for w, g, x, (_, n, ce, c0, cc) in zip(want, got, values, cases):
            assert torch.equal(w, g)    # bit-exact, as every decode test here
            assert torch.equal(g.cpu(), _expected_slice(x, n, ce, c0, cc))   # and equal to the encoded values


def test_noalloc_call_allocates_no_device_memory():
    cases, values = _cases(500, with_values=True)
    outs = _outputs(cases)
    rc, _ = _noalloc(cases, outs)             # warm-up: resolves the scratch address once
    assert rc == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        rc, st = _noalloc(cases, outs)
        assert rc == 0 and st == [0] * len(cases)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    for o, x, (_, n, ce, c0, cc) in zip(outs, values, cases):
        assert torch.equal(o.cpu(), _expected_slice(x, n, ce, c0, cc))


def test_noalloc_rejects_more_tensors_than_its_scratch_holds():
    from bigsmall_b200 import _lib
    cases = _cases(300)
    many = (cases * 2)[:9]
    rc, _ = _noalloc(many, _outputs(many))
    assert rc == _lib.BS_E_INVALID_ARG
    assert "at most 8 tensors" in _lib.last_error()


def test_noalloc_reports_corrupt_stream_and_recovers():
    from bigsmall_b200 import _lib
    cases = _cases(400)[:2]
    bad_blob = cases[0][0].clone()
    co = int(np.frombuffer(bad_blob[32:40].cpu().numpy().tobytes(), dtype="<u8")[0])
    bad_blob[co + 3] ^= 0x40                       # flip a lane state of chunk 0
    bad = [(bad_blob,) + cases[0][1:], cases[1]]
    rc, st = _noalloc(bad, _outputs(bad))
    assert rc == _lib.BS_E_CORRUPT and st[0] != 0 and st[1] == 0
    want = _with_plan(cases)
    got = _outputs(cases)
    rc, st = _noalloc(cases, got)
    assert rc == 0 and all(torch.equal(w, g) for w, g in zip(want, got))
