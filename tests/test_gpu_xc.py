"""GPU parity of the bf16_exp_chunked_v1 decoder and encoder (sm_100a).

Inputs are the reference's golden tensors (tests/golden) and seeded synthetic
tensors; the checker is the CPU oracle (oracle/bs_oracle.c) and the raw-byte
md5, the reference's own verification rule (bigsmall/verify.py:44-51).
Integer/byte work: every comparison is bit-exact.
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from tests.conftest import golden_bytes  # noqa: E402


def md5(b):
    return hashlib.md5(b).hexdigest()


def _dev(b: bytes):
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).cuda()


def _decode(blob: bytes, n: int, ce: int) -> bytes:
    from bigsmall_b200 import gpu
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    gpu.decode_xc_into(_dev(blob), out, ce)
    return out.cpu().view(torch.uint8).numpy().tobytes()


def _raw_bf16(n, seed=0, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("coder", [0, 1])
@pytest.mark.parametrize("prec", [10, 12])
@pytest.mark.parametrize("ce", [256, 4096, 65536])
def test_decode_golden_inputs(manifest, coder, prec, ce):
    for name, c in manifest["cases"].items():
        raw = golden_bytes(f"{name}.raw")
        blob = O.xc_encode(raw, coder, prec, ce)
        assert md5(_decode(blob, c["n"], ce)) == c["raw_md5"], (name, coder, prec, ce)


@pytest.mark.parametrize("n", [1, 31, 255, 256, 257, 4095, 4097, 65535, 65536, 65537, 300_001])
@pytest.mark.parametrize("coder", [0, 1])
def test_decode_ragged_sizes(n, coder):
    raw = _raw_bf16(n, seed=n).view(torch.uint8).numpy().tobytes()
    for ce in (256, 65536):
        blob = O.xc_encode(raw, coder, 12, ce)
        assert _decode(blob, n, ce) == raw, (n, coder, ce)


def test_device_encoder_matches_oracle_bytes(manifest):
    from bigsmall_b200 import gpu
    cases = [golden_bytes(f"{name}.raw") for name in manifest["cases"]]
    cases += [_raw_bf16(n, seed=n).view(torch.uint8).numpy().tobytes() for n in (1, 257, 65536, 200_003)]
    for raw in cases:
        n = len(raw) // 2
        x = torch.from_numpy(np.frombuffer(raw, dtype=np.int16).copy()).view(torch.bfloat16).cuda()
        for ce in (256, 65536):
            for prec in (11, 12):
                for coder, cid in (("rans", 0), ("tans", 1)):
                    d = gpu.encode_xc(x, coder=coder, prec=prec, chunk_elems=ce).cpu().numpy().tobytes()
                    assert d == O.xc_encode(raw, cid, prec, ce), (n, ce, prec, coder)


def test_full_size_config1_roundtrip_and_encoder_pin(manifest):
    """BASELINE config 1 at full size: device encode == oracle encode (md5),
    device decode == raw (md5)."""
    from bigsmall_b200 import gpu
    from tests.golden.make_golden import c1_tensor
    full = manifest["full_size"]["c1"]
    x = c1_tensor()
    raw = x.view(torch.uint8).numpy().tobytes()
    assert md5(raw) == full["raw_md5"]
    blob = gpu.encode_xc(x.cuda(), coder="rans")
    hb = blob.cpu().numpy().tobytes()
    assert md5(hb) == md5(O.xc_encode(raw, 0, 12, gpu.DEFAULT_CHUNK_ELEMS))
    out = torch.empty_like(x, device="cuda")
    gpu.decode_xc_into(blob, out, gpu.DEFAULT_CHUNK_ELEMS)
    assert md5(out.cpu().view(torch.uint8).numpy().tobytes()) == full["raw_md5"]
    assert len(hb) / len(raw) < 0.665   # exponent-rANS + raw plane ratio on config 1


def test_batched_plan_many_tensors():
    from bigsmall_b200 import gpu
    sizes = [4096, 1, 1_000_000, 65536 * 3 + 5, 777, 0, 123_456]
    xs = [_raw_bf16(n, seed=i, scale=0.01 * (i + 1)).cuda() for i, n in enumerate(sizes)]
    entries, outs = [], []
    for i, x in enumerate(xs):
        ce = 4096 if i % 2 else 65536
        blob = gpu.encode_xc(x, chunk_elems=ce) if x.numel() else torch.empty(0, dtype=torch.uint8, device="cuda")
        out = torch.empty_like(x)
        entries.append((blob, out, ce))
        outs.append(out)
    with gpu.XcPlan(entries) as plan:
        for _ in range(2):          # plans are reusable
            for o in outs:
                o.fill_(0)
            plan.run()
            for x, o in zip(xs, outs):
                assert torch.equal(x.view(torch.int16), o.view(torch.int16))


def test_corrupt_blobs_raise_without_fault():
    from bigsmall_b200 import gpu
    from bigsmall_b200.exceptions import BsCorruptError
    x = _raw_bf16(100_000, seed=3)
    raw = x.view(torch.uint8).numpy().tobytes()
    good = O.xc_encode(raw, 0, 12, 4096)
    co = struct.unpack_from("<Q", good, 32)[0]
    variants = {}
    b = bytearray(good); b[0] ^= 1; variants["magic"] = (bytes(b), 0x01)
    b = bytearray(good); b[64] ^= 0x10; variants["freq"] = (bytes(b), 0x02)
    b = bytearray(good); struct.pack_into("<I", b, 576 + 4, 0); variants["chunk_table"] = (bytes(b), 0x04)
    b = bytearray(good); b[co + 3] ^= 0x40; variants["lane_state"] = (bytes(b), 0x18)
    b = bytearray(good); b[co + 200] ^= 0xFF; variants["words"] = (bytes(b), 0x18)
    for name, (blob, bits) in variants.items():
        out = torch.empty(100_000, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(BsCorruptError) as ei:
            gpu.decode_xc_into(_dev(blob), out, 4096)
        st = ei.value.device_status[0]
        assert st and (st & bits), (name, hex(st))
    # the context is still healthy afterwards
    assert _decode(good, 100_000, 4096) == raw
    with pytest.raises(BsCorruptError):
        gpu.decode_xc_into(_dev(good[:-16]), torch.empty(100_000, dtype=torch.bfloat16, device="cuda"), 4096)
    with pytest.raises(ValueError):
        gpu.decode_xc_into(_dev(good), torch.empty(100_000, dtype=torch.bfloat16, device="cuda"), 1000)
