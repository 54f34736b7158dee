"""GPU parity of the bf16_parallel_v1 decoder against the reference's own blobs.

tests/golden holds blobs minted by the reference encoder
(bigsmall/codecs/bf16_parallel.py:186-259); the device decode must equal the
reference decode (bigsmall/codecs/bf16_parallel.py:262-352) byte for byte, as
the reference's only GPU test demands of its Triton path
(tests/test_gpu_kernel.py:37-51).
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from tests.conftest import golden_bytes  # noqa: E402


def md5(b):
    return hashlib.md5(b).hexdigest()


def _gpu_par(blob: bytes, n: int) -> bytes:
    from bigsmall_b200 import gpu
    d = torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy()).cuda() if blob else torch.empty(0, dtype=torch.uint8, device="cuda")
    out = torch.empty(max(n, 1), dtype=torch.bfloat16, device="cuda")
    gpu.decode_par_into(blob, d, out, n)
    return out[:n].cpu().view(torch.uint8).numpy().tobytes()


@pytest.mark.parametrize("key", ["par1", "par32", "par128"])
def test_reference_blobs(manifest, key):
    for name, c in manifest["cases"].items():
        b = c["blobs"][key]
        got = _gpu_par(golden_bytes(b["file"]), c["n"])
        assert md5(got) == b["decoded_md5"], (name, key)


@pytest.mark.parametrize("n,ns", [(1 << 18, 64), (1 << 20, 128), (1 << 20, 1), (300_001, 256)])
def test_gaussian(n, ns):
    """reference tests/test_gpu_kernel.py:37-51 shape (n=2^18, N=64) and more"""
    g = torch.Generator().manual_seed(ns)
    raw = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).view(torch.uint8).numpy().tobytes()
    blob = O.par_encode(raw, ns)
    assert _gpu_par(blob, n) == raw == O.par_decode(blob, n)


def test_errors_mirror_reference():
    from bigsmall_b200.exceptions import BsCorruptError
    raw = golden_bytes("gauss_8k.raw")
    blob = O.par_encode(raw, 32)
    with pytest.raises(BsCorruptError, match="bad magic"):
        _gpu_par(b"XXXX" + blob[4:], 8192)
    with pytest.raises(BsCorruptError, match="count mismatch"):
        _gpu_par(blob, 8191)
    bad = bytearray(blob)
    bad[10] = 13    # precision_se field
    with pytest.raises(BsCorruptError, match="precision"):
        _gpu_par(bytes(bad), 8192)
    with pytest.raises(BsCorruptError):
        _gpu_par(blob[:100], 8192)
    assert _gpu_par(b"", 0) == b""


def test_batched_serial_plan_mixes_parallel_and_legacy_blobs(manifest):
    """Every golden case as bf16_parallel_v1 (N = 1, 32, 128), bf16_se_single_kernel
    and bf16_se_tans blobs, all in ONE serial-format plan (BS_SE_PARALLEL next
    to the legacy codecs): all streams run concurrently, every output is the
    reference's decode."""
    from bigsmall_b200 import gpu
    kinds = (("par1", "bf16_parallel_v1"), ("par32", "bf16_parallel_v1"), ("par128", "bf16_parallel_v1"),
             ("sk", "bf16_se_single_kernel"), ("tans", "bf16_se_tans"))
    entries, want = [], []
    for name, c in manifest["cases"].items():
        raw = golden_bytes(f"{name}.raw")
        for key, codec in kinds:
            blob = golden_bytes(c["blobs"][key]["file"])
            d = (torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy()).cuda() if blob
                 else torch.empty(0, dtype=torch.uint8, device="cuda"))
            o = torch.empty(max(c["n"], 1), dtype=torch.int16, device="cuda")
            entries.append((codec, blob, d, o, c["n"]))
            want.append(raw)
    with gpu.SePlan(entries) as p:
        for _ in range(2):      # plans are reusable
            for e in entries:
                e[3].fill_(0)
            p.run()
            for (codec, _, _, o, n), raw in zip(entries, want):
                assert o[:n].cpu().view(torch.uint8).numpy().tobytes() == raw, codec


def test_many_parallel_tensors_take_the_grouped_schedule():
    """16 bf16_parallel_v1 tensors of 2^20 values (N = 128) in one serial-stream
    plan: 2,048 slice streams sharing 16 (sign,exp) tables plus their bucket
    streams, about 32M symbols -- far more than the job kernel's CTA slots can
    hold one stream each, so the plan's cost model runs table-sharing streams
    one per warp.  Every output must equal the reference decode."""
    from bigsmall_b200 import gpu
    n = 1 << 20
    raws, entries = [], []
    for k in range(16):
        g = torch.Generator().manual_seed(100 + k)
        raw = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).view(torch.uint8).numpy().tobytes()
        blob = O.par_encode(raw, 128)
        d = torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy()).cuda()
        entries.append(("bf16_parallel_v1", blob, d, torch.empty(n, dtype=torch.int16, device="cuda"), n))
        raws.append(raw)
    with gpu.SePlan(entries) as p:
        p.run()
    for (_, _, _, o, _), raw in zip(entries, raws):
        assert o.cpu().view(torch.uint8).numpy().tobytes() == raw
