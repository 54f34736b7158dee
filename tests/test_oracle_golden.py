"""Pin the CPU oracle against the reference's own golden vectors.

The fixtures under tests/golden/ were minted by tests/golden/make_golden.py
from the reference codecs (BigSmall bigsmall/codecs/rans.py,
bf16_parallel.py, single_kernel.py, bf16_tans.py).  The oracle must
reproduce every reference blob byte-for-byte when encoding and every raw
tensor when decoding; only then is it trusted as the checker for the CUDA
decoders.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import golden_bytes


def md5(b: bytes) -> str:
    return hashlib.md5(b).hexdigest()


def _cases(manifest):
    for name, c in sorted(manifest["cases"].items()):
        yield name, c


def test_golden_inputs_intact(manifest):
    for name, c in _cases(manifest):
        raw = golden_bytes(f"{name}.raw")
        assert md5(raw) == c["raw_md5"], name
        for key, b in c["blobs"].items():
            assert md5(golden_bytes(b["file"])) == b["md5"], (name, key)


@pytest.mark.parametrize("key", ["par1", "par32", "par128", "sk", "tans"])
def test_oracle_decodes_reference_blobs(manifest, key):
    dec = {"sk": O.sk_decode, "tans": O.tans_decode}.get(key, O.par_decode)
    for name, c in _cases(manifest):
        b = c["blobs"][key]
        out = dec(golden_bytes(b["file"]), c["n"])
        assert md5(out) == b["decoded_md5"] == c["raw_md5"], (name, key)


@pytest.mark.parametrize("key", ["par1", "par32", "par128", "sk", "tans"])
def test_oracle_encoder_matches_reference_bytes(manifest, key):
    for name, c in _cases(manifest):
        raw = golden_bytes(f"{name}.raw")
        if key == "sk":
            blob = O.sk_encode(raw)
        elif key == "tans":
            blob = O.tans_encode(raw)
        else:
            blob = O.par_encode(raw, int(key[3:]))
        assert md5(blob) == c["blobs"][key]["md5"], (name, key, len(blob), c["blobs"][key]["len"])


def test_rans_stream_vectors(manifest):
    """rans.py encode_stream/decode_stream, including the end-of-data quirk
    (rans.py:196-202): truncated streams decode exactly as the reference."""
    for v in manifest["rans_vectors"]:
        syms = np.frombuffer(bytes.fromhex(v["symbols_hex"]), dtype="<u2").astype(np.int32)
        freqs = np.array(v["freqs"], dtype=np.uint32)
        counts = np.bincount(syms, minlength=v["alphabet"]).astype(np.int64)
        assert (O.quantise_ref(counts, v["M"]) == freqs).all()
        data = bytes.fromhex(v["stream_hex"])
        assert O.rans_encode(syms, freqs, v["M"]) == data
        dec = O.rans_decode(data, v["n"], freqs, v["M"])
        assert (dec.astype(np.int64) == syms.astype(np.int64)).all()
        for cut in (1, 3):
            k = f"decode_cut{cut}_hex"
            if k in v:
                dd = O.rans_decode(data[:-cut], v["n"], freqs, v["M"])
                assert dd.astype("<u2").tobytes().hex() == v[k], (v["n"], cut)


def c1_raw() -> bytes:
    from tests.golden.make_golden import c1_tensor
    import torch
    return c1_tensor().contiguous().view(torch.uint8).numpy().tobytes()


def test_full_size_config1_pins(manifest):
    """BASELINE config 1 (4096x4096, seed 0): the oracle's single-kernel and
    tans encoders reproduce the reference blobs' md5 at full size."""
    full = manifest["full_size"]["c1"]
    raw = c1_raw()
    assert md5(raw) == full["raw_md5"]
    blob = O.sk_encode(raw)
    assert (len(blob), md5(blob)) == (full["sk"]["len"], full["sk"]["md5"])
    assert md5(O.sk_decode(blob, full["n"])) == full["raw_md5"]
    blob = O.tans_encode(raw)
    assert (len(blob), md5(blob)) == (full["tans"]["len"], full["tans"]["md5"])


def test_malformed_blobs_raise(manifest):
    c = manifest["cases"]["gauss_8k"]
    blob = golden_bytes(c["blobs"]["par32"]["file"])
    with pytest.raises(O.OracleError):
        O.par_decode(b"XXXX" + blob[4:], c["n"])
    with pytest.raises(O.OracleError):
        O.par_decode(blob, c["n"] + 1)
    with pytest.raises(O.OracleError):
        O.par_decode(blob[:40], c["n"])
    sk = golden_bytes(c["blobs"]["sk"]["file"])
    with pytest.raises(O.OracleError):
        O.sk_decode(sk, c["n"] - 1)
    with pytest.raises(O.OracleError):
        O.sk_decode(sk[: len(sk) // 2], c["n"])
