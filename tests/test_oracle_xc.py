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


@pytest.mark.parametrize("coder", [0, 1, 2])
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


@pytest.mark.parametrize("coder", [0, 1, 2])
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


def _u16(n, seed):
    return np.random.default_rng(seed).integers(0, 1 << 16, n, dtype=np.uint16).tobytes()


@pytest.mark.parametrize("n", [1, 2, 3, 255, 256, 257, 4095, 4097, 65537])
def test_xc_pair_coder_escapes_and_ragged_tails(n):
    """Coder 2 codes exponent pairs inside a 15-wide window, escaping the rest
    byte by byte; uniformly random words put most exponents outside it."""
    for raw in (_u16(n, n), (np.random.default_rng(n).standard_normal(n).astype(np.float32).view(np.uint32)
                             >> 16).astype(np.uint16).tobytes()):
        for ce in (256, 4096):
            blob = O.xc_encode(raw, 2, 12, ce)
            assert blob[6] == 2
            assert O.xc_decode(blob, n) == raw, (n, ce)


def test_xc_pair_coder_window_and_record_layout():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal(50000) * 0.02).astype(np.float32)
    raw = (w.view(np.uint32) >> 16).astype(np.uint16)
    blob = O.xc_encode(raw.tobytes(), 2, 12, 4096)
    e_lo = struct.unpack_from("<I", blob, 28)[0]
    ex = (raw >> 7) & 0xFF
    hist = np.bincount(ex, minlength=256)
    win = [int(hist[w:w + 15].sum()) for w in range(242)]
    assert e_lo == int(np.argmax(win))                     # first maximal window
    co = struct.unpack_from("<Q", blob, 32)[0]
    ends = np.frombuffer(blob, dtype="<u4", count=14, offset=576)
    n_esc_total = 0
    for k in range(13):
        rec = co + 16 * int(ends[k])
        size = 16 * int(ends[k + 1] - ends[k])
        nw, ne, z0, z1 = struct.unpack_from("<IIII", blob, rec + 128)
        assert (z0, z1) == (0, 0)
        assert 144 + 2 * nw + ne <= size < 144 + 2 * nw + ne + 16
        n_esc_total += ne
    outside = int(((ex < e_lo) | (ex > e_lo + 14)).sum())
    assert n_esc_total == outside


def test_xc_pair_coder_bad_escape_count_detected():
    raw = _u16(20000, 9)
    blob = bytearray(O.xc_encode(raw, 2, 12, 4096))
    co = struct.unpack_from("<Q", blob, 32)[0]
    ne = struct.unpack_from("<I", blob, co + 132)[0]
    assert ne > 0
    struct.pack_into("<I", blob, co + 132, ne - 1)
    with pytest.raises(O.OracleError):
        O.xc_decode(bytes(blob), 20000)
    bad = bytearray(O.xc_encode(raw, 2, 12, 4096))
    struct.pack_into("<I", bad, 28, 300)                  # window base out of range
    with pytest.raises(O.OracleError):
        O.xc_decode(bytes(bad), 20000)


def _special(kind: str, n: int) -> bytes:
    rng = np.random.default_rng(n)
    if kind == "zeros":
        w = np.zeros(n, np.uint16)
    elif kind == "nan_inf":
        w = rng.choice(np.array([0x7F80, 0xFF80, 0x7FC0, 0xFFFF, 0x7F81], np.uint16), n)
    elif kind == "subnormal":
        w = (rng.integers(0, 0x80, n) | (rng.integers(0, 2, n) << 15)).astype(np.uint16)
    elif kind == "top_exponents":      # exponents 240..255: window base at its maximum (241)
        e = rng.integers(240, 256, n)
        w = ((rng.integers(0, 2, n) << 15) | (e << 7) | rng.integers(0, 128, n)).astype(np.uint16)
    elif kind == "many_rare":          # every exponent present, two dominant ones: at low precision
        # the rare symbols' floor of 1 overshoots M and the excess is taken
        # from more than one symbol
        e = np.where(rng.random(n) < 0.5, 120, 121)
        k = min(n, 512)
        e[:k] = np.arange(k) % 256
        w = ((e << 7) | rng.integers(0, 128, n)).astype(np.uint16)
    else:                              # two far-apart exponent clusters: many escapes
        e = np.where(rng.random(n) < 0.5, rng.integers(1, 8, n), rng.integers(200, 230, n))
        w = ((e << 7) | rng.integers(0, 128, n)).astype(np.uint16)
    return w.tobytes()


@pytest.mark.parametrize("kind", ["zeros", "nan_inf", "subnormal", "top_exponents", "two_clusters", "many_rare"])
@pytest.mark.parametrize("coder", [0, 1, 2])
@pytest.mark.parametrize("prec", [8, 10, 12])
def test_xc_special_value_distributions(kind, coder, prec):
    for n in (1, 300, 70_001):
        raw = _special(kind, n)
        blob = O.xc_encode(raw, coder, prec, 4096)
        assert O.xc_decode(blob, n) == raw, (kind, coder, prec, n)


# ---- state groups per chunk (format version 2) -----------------------------
@pytest.mark.parametrize("coder", [0, 1, 2])
@pytest.mark.parametrize("chunk,groups", [(4096, 2), (65536, 8), (65536, 256), (1 << 20, 32), (1 << 21, 64)])
def test_xc_groups_roundtrip_and_layout(manifest, coder, chunk, groups):
    """A chunk of `chunk` values in `groups` state groups: the blob decodes
    exactly, and everything past the header equals the one-group blob with
    chunk / groups values per chunk (the group records, offset table, plane
    and frequency table are the same bytes)."""
    for name, c in manifest["cases"].items():
        raw = golden_bytes(f"{name}.raw")
        blob = O.xc_encode(raw, coder, 12, chunk, groups)
        assert md5(O.xc_decode(blob, c["n"])) == c["raw_md5"], (name, coder, chunk, groups)
        one = O.xc_encode(raw, coder, 12, chunk // groups)
        assert blob[64:] == one[64:] and len(blob) == len(one)
        ver = struct.unpack_from("<H", blob, 4)[0]
        n, ce, nc = struct.unpack_from("<QII", blob, 8)
        g, zero = struct.unpack_from("<II", blob, 56)
        assert (ver, ce, nc, g, zero) == (2, chunk, -(-c["n"] // chunk), groups, 0)


@pytest.mark.parametrize("coder", [0, 2])
def test_xc_groups_header_checked(coder):
    rng = np.random.default_rng(7)
    raw = (rng.standard_normal(70001).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    blob = O.xc_encode(raw, coder, 12, 65536, 8)
    assert O.xc_decode(blob, 70001) == raw
    for off, val in ((56, 0), (56, 3), (56, 16), (60, 1), (16, 65536 + 256), (20, 1), (4, 3)):
        bad = bytearray(blob)
        struct.pack_into("<H" if off == 4 else "<I", bad, off, val)
        with pytest.raises(O.OracleError):
            O.xc_decode(bytes(bad), 70001)
    with pytest.raises(O.OracleError):       # chunk / groups below 256 values
        O.xc_encode(raw, coder, 12, 4096, 32)
    with pytest.raises(O.OracleError):       # chunk not a multiple of groups
        O.xc_encode(raw, coder, 12, 65536, 3)


def _product_model_freqs(raw: np.ndarray, prec: int = 12) -> tuple[int, np.ndarray]:
    """The pair coder's frequency rule restated in numpy: the exponent
    histogram counts every value, or for n >= 2^20 the 2048-value blocks whose
    index is a multiple of 8; window = first maximal 15-exponent window;
    window-index marginals c(a) of the s counted values; m(a) =
    max(1, c(a) * 2^16 // s) for c(a) > 0, else 1 if sampled, 0 if not;
    counts m(a) * m(b), plus 1 at (a of the last value, 0) for odd n; then the
    format's quantisation."""
    n = raw.size
    ex = (raw >> 7) & 0xFF
    sampled = n >= 1 << 20
    counted = ex[((np.arange(n) >> 11) & 7) == 0] if sampled else ex
    hist = np.bincount(counted, minlength=256).astype(np.int64)
    e_lo = int(np.argmax([hist[w:w + 15].sum() for w in range(242)]))
    c = np.zeros(16, np.int64)
    c[:15] = hist[e_lo:e_lo + 15]
    c[15] = counted.size - c[:15].sum()
    m = np.where(c > 0, np.maximum(1, (c << 16) // counted.size), 1 if sampled else 0)
    pc = np.outer(m, m).reshape(-1)
    if n % 2:
        d = int(ex[-1]) - e_lo
        pc[(d if 0 <= d <= 14 else 15) * 16] += 1
    return e_lo, O.xc_quantise(pc, prec)


@pytest.mark.parametrize("seed,n", [(0, 50_000), (1, 50_001), (2, 1), (3, 255), (4, 70_001),
                                    (5, (1 << 20) - 1), (6, 1 << 20), (7, (1 << 20) + 12_345), (8, 3 << 20)])
def test_xc_pair_coder_frequencies_follow_the_product_model(seed, n):
    """Coder 2 quantises m(a) * m(b) from the exponent histogram alone (no pass
    over the pairs; an eighth of the blocks from 2^20 values on); its header's
    window and frequency table match a numpy restatement of that rule, for
    normal, wide-range and odd-length inputs on both sides of the threshold."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(n) * np.exp(rng.standard_normal(n) * (3 if seed % 2 else 0.3))).astype(np.float32)
    raw = (w.view(np.uint32) >> 16).astype(np.uint16)
    for prec in (10, 12):
        blob = O.xc_encode(raw.tobytes(), 2, prec, 4096)
        e_lo, want = _product_model_freqs(raw, prec)
        assert struct.unpack_from("<I", blob, 28)[0] == e_lo
        assert np.array_equal(np.frombuffer(blob, dtype="<u2", count=256, offset=64), want), (seed, n, prec)
        assert O.xc_decode(blob, n) == raw.tobytes()


def test_xc_pair_coder_sample_unlike_the_rest_still_round_trips():
    """From 2^20 values on the pair coder's statistics come from every eighth
    2048-value block.  When those blocks are all zeros and the rest are normal
    weights, every other value escapes the window: the ratio suffers, the round
    trip does not."""
    n = (1 << 20) + 4097
    rng = np.random.default_rng(11)
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    raw = (w.view(np.uint32) >> 16).astype(np.uint16)
    raw[((np.arange(n) >> 11) & 7) == 0] = 0
    blob = O.xc_encode(raw.tobytes(), 2, 12, 32768)
    assert struct.unpack_from("<I", blob, 28)[0] == 0            # window at the zeros' exponent
    assert O.xc_decode(blob, n) == raw.tobytes()
    assert len(blob) > 2 * n                                      # most exponents escaped
