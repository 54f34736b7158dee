"""Container format (BigSmall bigsmall/container.py layout) and partitioning, CPU only."""
from __future__ import annotations

import json
import math
import struct

import pytest

from bigsmall_b200 import container as C
from bigsmall_b200.exceptions import BigSmallVersionError


def test_writer_roundtrip_and_alignment(tmp_path):
    w = C.ContainerWriter()
    w.add("a", [3], "BF16", "raw", b"\x01\x02" * 3, "m1")
    w.add("b", [5], "BF16", "bf16_exp_chunked_v1", b"x" * 37, "m2", {"chunk_elems": 256})
    w.add("c", [5], "BF16", "tied_ref", b"", "m2", {"tied_to": "b"})
    w.add("d", [2, 2], "F32", "raw", b"\0" * 16, "m3")
    buf = w.to_bytes()
    header, off = C.parse_header(buf)
    assert buf[:4] == b"BGSM" and struct.unpack_from("<H", buf, 4)[0] == 2   # v2: new codec present
    assert header["tensor_count"] == 4 and header["_format_version"] == 2
    for t in header["tensors"]:
        if t["codec"] != "tied_ref":
            assert t["offset"] % 16 == 0
    data = memoryview(buf)[off:]
    blobs = {t["name"]: bytes(b) for t, b in C.iter_blobs(header, data)}
    assert blobs["a"] == b"\x01\x02" * 3 and blobs["b"] == b"x" * 37 and blobs["d"] == b"\0" * 16
    p = tmp_path / "m.bs"
    w.write(p)
    h2, off2 = C.read_header(p)
    assert h2["tensors"] == header["tensors"] and off2 == off
    assert C.read_blob(p, h2, off2, 1) == b"x" * 37
    info = C.info(p)
    assert info["tensor_count"] == 4 and info["codec_stats"]["raw"] == 2


def test_version_and_magic_errors(tmp_path):
    hb = json.dumps({"tensors": [], "tensor_count": 0}).encode()
    bad = b"BGSM" + struct.pack("<H", 9) + struct.pack("<I", len(hb)) + hb
    with pytest.raises(BigSmallVersionError):
        C.parse_header(bad)
    with pytest.raises(ValueError):
        C.parse_header(b"NOPE" + bad[4:])
    C.write_container(tmp_path / "v1.bs", {"tensors": [], "tensor_count": 0}, b"")
    assert C.read_header(tmp_path / "v1.bs")[0]["_format_version"] == 1


def test_v1_files_read():
    """A reference-written (v1, unaligned offsets) container parses identically."""
    hdr = {"format": "bf16", "tensor_count": 1,
           "tensors": [{"name": "w", "shape": [2], "dtype": "BF16", "codec": "raw", "special": None,
                        "compressed_bytes": 4, "offset": 0, "md5": "", "extra": None}]}
    hb = json.dumps(hdr, separators=(",", ":")).encode()
    buf = b"BGSM" + struct.pack("<H", 1) + struct.pack("<I", len(hb)) + hb + b"\x01\x02\x03\x04"
    h, off = C.parse_header(buf)
    assert h["tensors"][0]["name"] == "w" and buf[off:] == b"\x01\x02\x03\x04"


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_partition_covers_container_once(world):
    import bench
    from bigsmall_b200.sharding import partition
    tensors = bench.llama3_8b_tensors()
    owned, load = partition(tensors, world, 65536)
    assert max(load) - min(load) <= 65536
    seen = {}
    for r in owned:
        assert len({n for n, _, _ in r}) == len(r)
        for name, c0, cc in r:
            seen.setdefault(name, []).append((c0, cc))
    for name, shape, _ in tensors:
        nc = -(-math.prod(shape) // 65536)
        pos = 0
        for c0, cc in sorted(seen[name]):
            assert c0 == pos
            pos = c0 + (cc or nc)
        assert pos == nc


def test_top_level_names_follow_the_reference():
    import bigsmall_b200 as b
    for name in ("decompress", "load", "verify", "info", "StreamingLoader", "BigSmallStreamingModel",
                 "CompressedKVCache", "BigSmallVersionError"):
        assert callable(getattr(b, name)), name


def test_owned_for_header_mixed_chunk_sizes():
    """Per-tensor chunk sizes from the header; every chunk has one owner and
    rank loads differ by at most the largest chunk."""
    from bigsmall_b200.sharding import owned_for, partition_chunks
    sizes = [(f"t{i}", n, ce) for i, (n, ce) in
             enumerate([(5_000_000, 32768), (123_457, 65536), (40_000_000, 32768), (4096, 256), (9_999_999, 65536)])]
    hdr = {"tensors": [{"name": nm, "shape": [n], "codec": "bf16_exp_chunked_v1", "extra": {"chunk_elems": ce}}
                       for nm, n, ce in sizes] + [
        {"name": "raw", "shape": [7], "codec": "raw", "extra": {}},
        {"name": "par", "shape": [3000, 1000], "codec": "bf16_parallel_v1", "extra": {}},
        {"name": "empty", "shape": [0], "codec": "raw", "extra": {}},
        {"name": "tied", "shape": [7], "codec": "tied_ref", "extra": {"tied_to": "raw"}}]}
    for world in (1, 2, 3, 5, 8):
        owned = [owned_for(hdr, r, world) for r in range(world)]
        _, load = partition_chunks(sizes, world)
        assert max(load) - min(load) <= 65536
        for nm, n, ce in sizes:
            nc = -(-n // ce)
            parts = sorted((c0, cc or nc) for r in owned for name, c0, cc in r if name == nm)
            pos = 0
            for c0, cc in parts:
                assert c0 == pos
                pos += cc
            assert pos == nc
        for whole in ("raw", "par", "empty"):   # unsplittable tensors: exactly one owner, whole
            assert [(c0, cc) for r in owned for name, c0, cc in r if name == whole] == [(0, 0)]
        assert all(name != "tied" for r in owned for name, _, _ in r)
    with pytest.raises(ValueError):
        owned_for(hdr, 2, 2)


def test_version_error_messages_follow_the_reference():
    """Message shape of BigSmallVersionError for a future container version, an
    unknown codec and direct construction (reference tests/test_version_errors.py:12-71)."""
    import bigsmall_b200
    from bigsmall_b200.decoder import _decode_blob
    assert issubclass(bigsmall_b200.BigSmallVersionError, Exception)
    hb = b"{}"
    with pytest.raises(BigSmallVersionError) as ei:
        C.parse_header(b"BGSM" + struct.pack("<H", 99) + struct.pack("<I", len(hb)) + hb)
    assert "pip install --upgrade bigsmall" in str(ei.value) and "requires bigsmall >= 2.4.0" in str(ei.value)
    meta = {"name": "x", "shape": [4], "dtype": "BF16", "codec": "future_codec_v9", "special": None,
            "compressed_bytes": 8, "offset": 0, "md5": "0" * 32, "extra": None}
    with pytest.raises(BigSmallVersionError) as ei:
        _decode_blob(meta, b"\x00" * 8)
    assert "pip install --upgrade bigsmall" in str(ei.value) and "future_codec_v9" in str(ei.value)
    msg = str(BigSmallVersionError(required="3.0.0", installed="2.4.0", detail="hypothetical"))
    for part in ("requires bigsmall >= 3.0.0", "you have 2.4.0", "pip install --upgrade bigsmall", "hypothetical"):
        assert part in msg
