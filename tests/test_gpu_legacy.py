"""GPU decode of the legacy serial formats bf16_se_single_kernel and
bf16_se_tans (sm_100a), against the reference-minted golden blobs and the
oracle (bigsmall/codecs/single_kernel.py:432-613, bigsmall/codecs/bf16_tans.py:
121-167 + numba_rans.py:168-217).  Byte work: every comparison is bit-exact."""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from tests.conftest import golden_bytes  # noqa: E402

NAMES = {"sk": "bf16_se_single_kernel", "tans": "bf16_se_tans"}


def _dev(b: bytes):
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).cuda()


def _decode(kind: str, blob: bytes, n: int) -> bytes:
    from bigsmall_b200 import gpu
    out = torch.empty(max(n, 1), dtype=torch.int16, device="cuda")
    gpu.decode_se_into(NAMES[kind], blob, _dev(blob) if blob else None, out, n)
    return out[:n].cpu().numpy().tobytes()


@pytest.mark.parametrize("kind", ["sk", "tans"])
def test_golden_blobs(manifest, kind):
    for name, c in manifest["cases"].items():
        b = c["blobs"][kind]
        blob = golden_bytes(b["file"])
        got = _decode(kind, blob, c["n"])
        assert hashlib.md5(got).hexdigest() == c["raw_md5"] == b["decoded_md5"], name


@pytest.mark.parametrize("kind", ["sk", "tans"])
def test_full_size_config1(manifest, kind):
    from tests.golden.make_golden import c1_tensor
    full = manifest["full_size"]["c1"]
    raw = c1_tensor().view(torch.uint8).numpy().tobytes()
    blob = getattr(O, f"{kind}_encode")(raw)
    assert hashlib.md5(blob).hexdigest() == full[kind]["md5"]       # the reference's own blob bytes
    got = _decode(kind, blob, full["n"])
    assert hashlib.md5(got).hexdigest() == full["raw_md5"]


@pytest.mark.parametrize("kind", ["sk", "tans"])
@pytest.mark.parametrize("n", [1, 2, 31, 4097, 100_003])
def test_oracle_blobs_ragged(kind, n):
    rng = np.random.default_rng(n)
    w = (rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 2)).astype(np.float32)
    raw = (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    blob = getattr(O, f"{kind}_encode")(raw)
    assert _decode(kind, blob, n) == raw == getattr(O, f"{kind}_decode")(blob, n)


@pytest.mark.parametrize("kind", ["sk", "tans"])
def test_corrupt_stream_reports_without_fault(kind):
    from bigsmall_b200 import gpu
    from bigsmall_b200.exceptions import BsCorruptError
    n = 50_000
    rng = np.random.default_rng(7)
    raw = (rng.standard_normal(n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    blob = bytearray(getattr(O, f"{kind}_encode")(raw))
    # damage the (sign,exp) stream: its decoded exponent histogram no longer
    # matches the recorded bucket sizes
    n_se_nz = struct.unpack_from("<H", blob, 4)[0]
    at = 6 + 6 * n_se_nz + 8 + 64
    for k in range(8):
        blob[at + k] ^= 0xA5
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    with pytest.raises(BsCorruptError):
        gpu.decode_se_into(NAMES[kind], bytes(blob), _dev(bytes(blob)), out, n)
    with pytest.raises(ValueError):
        gpu.decode_se_into(NAMES[kind], bytes(blob), _dev(bytes(blob)), out, n + 1)
    good = getattr(O, f"{kind}_encode")(raw)
    assert _decode(kind, good, n) == raw          # the context is still usable


def test_registry_dispatch_and_loader():
    from bigsmall_b200 import codec_registry, decoder, gpu
    from bigsmall_b200.container import ContainerWriter
    from bigsmall_b200.loader import ContainerImage, DeviceLoader
    rng = np.random.default_rng(11)
    tensors = {}
    w = ContainerWriter(fmt="bf16")
    for i, (kind, n) in enumerate((("sk", 70_001), ("tans", 33_333), ("xc", 65_536 * 2 + 9), ("par", 20_000))):
        v = (rng.standard_normal(n).astype(np.float32) * 0.02).view(np.uint32) >> 16
        raw = v.astype(np.uint16).tobytes()
        name = f"model.layers.{i}.w"
        if kind == "xc":
            blob = O.xc_encode(raw, 2, 12, 65536)
            w.add(name, [n], "BF16", "bf16_exp_chunked_v1", blob, "", gpu.xc_extras(65536, "pair"))
        elif kind == "par":
            w.add(name, [n], "BF16", "bf16_parallel_v1", O.par_encode(raw, 32), "", {"n_streams": 32})
        else:
            blob = getattr(O, f"{kind}_encode")(raw)
            w.add(name, [n], "BF16", NAMES[kind], blob, "", {})
            _, dec = codec_registry.get_codec(NAMES[kind])
            assert dec(blob, {}, n) == raw
            assert decoder._decode_blob({"codec": NAMES[kind], "shape": [n], "extra": {}}, blob) == raw
        tensors[name] = raw
    img = ContainerImage.from_bytes(w.to_bytes())
    ld = DeviceLoader(img, device=0, group_bytes=50_000)
    for _ in range(2):
        out = ld.run()
        for name, raw in tensors.items():
            assert out[name].cpu().view(torch.uint8).numpy().tobytes() == raw, name
    ld.close()
