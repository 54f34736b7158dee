"""Host-side framing of the legacy serial formats (bf16_se_single_kernel,
bf16_se_tans) through the C ABI's bs_se_parse: no device work, so it runs
on CPU.  The reference-minted golden blobs must parse into one (sign,exp)
stream plus one stream per exponent bucket; damaged framing must fail the
way the oracle's decoder fails (bigsmall/codecs/single_kernel.py:432-580,
bigsmall/codecs/bf16_tans.py:121-167)."""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import golden_bytes

CODECS = {"sk": 1, "tans": 2}


def _parse(kind: str, blob: bytes, n: int):
    from bigsmall_b200 import _lib
    L = _lib.load()
    out = ctypes.c_uint32()
    buf = ctypes.create_string_buffer(blob, len(blob)) if blob else None
    rc = L.bs_se_parse(CODECS[kind], buf, len(blob), n, ctypes.byref(out))
    return rc, out.value


def _n_buckets(raw: bytes) -> int:
    w = np.frombuffer(raw, dtype=np.uint16)
    return len(np.unique((w >> 7) & 0xFF)) if len(w) else 0


@pytest.mark.parametrize("kind", ["sk", "tans"])
def test_golden_blobs_parse(manifest, kind):
    for name, c in manifest["cases"].items():
        blob = golden_bytes(c["blobs"][kind]["file"])
        raw = golden_bytes(f"{name}.raw")
        rc, jobs = _parse(kind, blob, c["n"])
        assert rc == 0, (name, rc)
        assert jobs == 1 + _n_buckets(raw), (name, jobs)


@pytest.mark.parametrize("kind", ["sk", "tans"])
def test_damaged_framing_fails_like_the_oracle(kind):
    from bigsmall_b200 import _lib
    rng = np.random.default_rng(3)
    w = (rng.standard_normal(5000).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    raw = w.tobytes()
    blob = getattr(O, f"{kind}_encode")(raw)
    dec = getattr(O, f"{kind}_decode")
    assert _parse(kind, blob, 5000)[0] == 0
    # count mismatch
    assert _parse(kind, blob, 5001)[0] == _lib.BS_E_COUNT_MISMATCH
    with pytest.raises(O.OracleError):
        dec(blob, 5001)
    # truncated inside the header
    for cut in (3, 9, 40):
        assert _parse(kind, blob[:cut], 5000)[0] in (_lib.BS_E_TRUNCATED, _lib.BS_E_CORRUPT), cut
        with pytest.raises(O.OracleError):
            dec(blob[:cut], 5000)
    # SE symbol index out of range
    bad = bytearray(blob)
    struct.pack_into("<H", bad, 6, 600)
    assert _parse(kind, bytes(bad), 5000)[0] == _lib.BS_E_CORRUPT
    with pytest.raises(O.OracleError):
        dec(bytes(bad), 5000)
    # empty blob / zero weights: nothing to decode
    assert _parse(kind, b"", 0) == (0, 0)


def test_single_kernel_frequency_sum_enforced():
    from bigsmall_b200 import _lib
    rng = np.random.default_rng(4)
    raw = (rng.standard_normal(3000).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    blob = bytearray(O.sk_encode(raw))
    n_se_nz = struct.unpack_from("<H", blob, 4)[0]
    f0 = struct.unpack_from("<I", blob, 6 + 2 * n_se_nz)[0]
    struct.pack_into("<I", blob, 6 + 2 * n_se_nz, f0 + 1)      # SE frequencies now sum to 4097
    assert _parse("sk", bytes(blob), 3000)[0] == _lib.BS_E_CORRUPT
    with pytest.raises(O.OracleError):
        O.sk_decode(bytes(blob), 3000)


@pytest.mark.parametrize("key,ns", [("par1", 1), ("par32", 32), ("par128", 128)])
def test_golden_parallel_blobs_parse_in_serial_plans(manifest, key, ns):
    """bf16_parallel_v1 (BS_SE_PARALLEL in a serial-format batch): one (sign,
    exp) stream per non-empty slice k::N plus one per exponent bucket of the
    slice (bigsmall/codecs/bf16_parallel.py:262-352)."""
    from bigsmall_b200 import _lib
    L = _lib.load()
    for name, c in manifest["cases"].items():
        blob = golden_bytes(c["blobs"][key]["file"])
        w = np.frombuffer(golden_bytes(f"{name}.raw"), dtype=np.uint16)
        want = sum(1 + len(np.unique((w[k::ns] >> 7) & 0xFF)) for k in range(ns) if len(w[k::ns]))
        out = ctypes.c_uint32()
        buf = ctypes.create_string_buffer(blob, len(blob)) if blob else None
        rc = L.bs_se_parse(_lib.SE_PARALLEL, buf, len(blob), c["n"], ctypes.byref(out))
        assert rc == 0, (name, rc)
        assert out.value == (want if c["n"] else 0), (name, out.value, want)
        if c["n"]:
            assert L.bs_se_parse(_lib.SE_PARALLEL, buf, len(blob), c["n"] + 1,
                                 ctypes.byref(out)) == _lib.BS_E_COUNT_MISMATCH
