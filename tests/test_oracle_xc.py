"""CPU oracle of this project's bf16_exp_chunked_v1 format.

The format has no reference counterpart, so its parity anchor is the md5 of
the raw tensor bytes (the reference's own verification, bigsmall/verify.py:
44-51): encode -> decode must reproduce every input exactly, for every coder,
precision and chunk size, on the reference's edge-case fixtures.
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import golden_bytes


def md5(b):
    return hashlib.md5(b).hexdigest()


@pytest.mark.parametrize("coder", [0, 1])
@pytest.mark.parametrize("prec", [10, 11, 12])
@pytest.mark.parametrize("chunk", [256, 4096, 65536])
def test_xc_roundtrip_golden_inputs(manifest, coder, prec, chunk):
    for name, c in manifest["cases"].items():
        raw = golden_bytes(f"{name}.raw")
        blob = O.xc_encode(raw, coder, prec, chunk)
        assert md5(O.xc_decode(blob, c["n"])) == c["raw_md5"], (name, coder, prec, chunk)


def test_xc_header_fields():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(70000) * 0.02).astype(np.float32)
    raw = (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    blob = O.xc_encode(raw, 0, 12, 32768)
    assert blob[:4] == b"BSXC"
    ver, coder, prec = struct.unpack_from("<HBB", blob, 4)
    n, ce, nc, lanes = struct.unpack_from("<QIII", blob, 8)
    co, po, tot = struct.unpack_from("<QQQ", blob, 32)
    assert (ver, coder, prec, n, ce, nc, lanes) == (1, 0, 12, 70000, 32768, 3, 32)
    assert po == (576 + 4 * 4 + 15) // 16 * 16 and co == po + (70000 + 15) // 16 * 16
    assert tot == len(blob) and tot % 16 == 0
    freq = np.frombuffer(blob, dtype="<u2", count=256, offset=64)
    assert int(freq.sum()) == 4096 and int(freq.max()) < 4096


def test_xc_quantise_rules():
    c = np.zeros(256, np.int64)
    c[127] = 1000
    f = O.xc_quantise(c, 12)
    assert f[127] == 4095 and f[128] == 1 and f.sum() == 4096          # phantom symbol
    c = np.zeros(256, np.int64)
    c[[3, 4, 5]] = [1, 1, 10 ** 9]
    f = O.xc_quantise(c, 12)
    assert f[3] == 1 and f[4] == 1 and f[5] == 4094
    c = np.arange(256, dtype=np.int64)
    f = O.xc_quantise(c, 8)
    assert f.sum() == 256 and (f[1:] >= 1).all() and f[0] == 0


@pytest.mark.parametrize("coder", [0, 1])
def test_xc_corruption_detected(coder):
    rng = np.random.default_rng(1)
    raw = (rng.standard_normal(20000).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    blob = bytearray(O.xc_encode(raw, coder, 12, 4096))
    n = 20000
    with pytest.raises(O.OracleError):
        O.xc_decode(bytes(blob), n + 1)
    with pytest.raises(O.OracleError):
        O.xc_decode(bytes(blob[:-16]), n)
    bad = bytearray(blob)
    bad[0] = ord("X")
    with pytest.raises(O.OracleError):
        O.xc_decode(bytes(bad), n)
    # flip a lane state of chunk 0 -> final-state / stream check fails
    co = struct.unpack_from("<Q", blob, 32)[0]
    bad = bytearray(blob)
    bad[co + 5] ^= 0x5A
    with pytest.raises(O.OracleError):
        O.xc_decode(bytes(bad), n)
