"""``.bs`` container read/write (format-compatible with the reference).

Layout (BigSmall ``bigsmall/container.py:1-38``)::

    [4]  magic b"BGSM"
    [2]  u16 version (1 or 2; a v2 reader accepts v1)
    [4]  u32 header JSON length
    [N]  header JSON (utf-8): {"format", "mode", "model_type", "base_model",
         "tensor_count", "tensors": [{"name", "shape", "dtype", "codec",
         "special", "compressed_bytes", "offset", "md5", "extra"}], ...}
    [..] data section: blobs at their ``offset``

This writer keeps every blob 16-byte aligned inside the data section (the
offsets are explicit, so readers of the reference format are unaffected);
the device decoders read blobs with 16-byte vector loads.
"""
from __future__ import annotations

import io
import json
import struct
from pathlib import Path
from typing import Any, BinaryIO, Iterable, Optional

from .exceptions import BigSmallVersionError

MAGIC = b"BGSM"
FORMAT_VERSION_V1 = 1
FORMAT_VERSION_V2 = 2
SUPPORTED_VERSIONS = frozenset({FORMAT_VERSION_V1, FORMAT_VERSION_V2})
# codecs that need a v2 reader (bigsmall/encoder.py:484-488 promotes the same way)
V2_CODECS = {"bf16_sparsity_v1", "fp2_residual_v1", "bf16_parallel_v1", "bf16_exp_chunked_v1"}
BLOB_ALIGN = 16

DTYPE_BYTES = {
    "F32": 4, "float32": 4, "F16": 2, "float16": 2, "BF16": 2, "bfloat16": 2,
    "F8_E4M3": 1, "float8_e4m3fn": 1, "F8_E5M2": 1, "float8_e5m2": 1,
    "I64": 8, "int64": 8, "I32": 4, "int32": 4, "I16": 2, "int16": 2,
    "I8": 1, "int8": 1, "U8": 1, "uint8": 1, "BOOL": 1, "bool": 1,
}


def n_elements(shape) -> int:
    """Element count as the reference computes it (bigsmall/decoder.py:53)."""
    n = 1
    for d in shape or []:
        n *= int(d)
    return n if shape else 1


def parse_header(buf: bytes | memoryview) -> tuple[dict, int]:
    """Parse a container prefix; returns (header, data_offset).

    Mirrors bigsmall/container.py:85-116 read_header, including its errors.
    """
    mv = memoryview(buf)
    if len(mv) < 10 or bytes(mv[:4]) != MAGIC:
        raise ValueError(f"Not a BigSmall .bs file (magic={bytes(mv[:4])!r})")
    version, = struct.unpack_from("<H", mv, 4)
    if version not in SUPPORTED_VERSIONS:
        from . import __version__
        raise BigSmallVersionError(
            required="2.4.0", installed=__version__,
            detail=f"file uses container format v{version}; this build supports {sorted(SUPPORTED_VERSIONS)}")
    hlen, = struct.unpack_from("<I", mv, 6)
    if len(mv) < 10 + hlen:
        raise ValueError("truncated .bs header")
    header = json.loads(bytes(mv[10:10 + hlen]).decode("utf-8"))
    header["_format_version"] = version
    return header, 10 + hlen


def read_header(path) -> tuple[dict, int]:
    with open(path, "rb") as f:
        head = f.read(10)
        if len(head) < 10:
            raise ValueError("truncated .bs file")
        hlen, = struct.unpack_from("<I", head, 6)
        return parse_header(head + f.read(hlen))


def read_blob(path, header: dict, data_offset: int, tensor_idx: int) -> bytes:
    t = header["tensors"][tensor_idx]
    with open(path, "rb") as f:
        f.seek(data_offset + t["offset"])
        return f.read(t["compressed_bytes"])


class ContainerWriter:
    """Assemble a container from already-encoded blobs, keeping each blob
    16-byte aligned in the data section."""

    def __init__(self, fmt: str = "bf16", mode: str = "balanced", model_type: str = "llm"):
        self.meta = {"format": fmt, "mode": mode, "model_type": model_type, "base_model": None}
        self.tensors: list[dict] = []
        self.data = io.BytesIO()
        self.codec_stats: dict[str, int] = {}

    def add(self, name: str, shape, dtype: str, codec: str, blob: bytes, md5: str = "",
            extra: Optional[dict] = None, special: Optional[str] = None) -> dict:
        pad = (-self.data.tell()) % BLOB_ALIGN
        if pad and codec != "tied_ref":
            self.data.write(b"\0" * pad)
        off = self.data.tell()
        self.data.write(blob)
        entry = {"name": name, "shape": [int(s) for s in shape], "dtype": dtype, "codec": codec,
                 "special": special, "compressed_bytes": len(blob), "offset": off, "md5": md5,
                 "extra": extra or None}
        self.tensors.append(entry)
        self.codec_stats[codec] = self.codec_stats.get(codec, 0) + 1
        return entry

    def header(self) -> dict:
        h = dict(self.meta)
        h["tensor_count"] = len(self.tensors)
        h["tensors"] = self.tensors
        h["codec_stats"] = dict(self.codec_stats)
        return h

    def version(self) -> int:
        return FORMAT_VERSION_V2 if any(t["codec"] in V2_CODECS for t in self.tensors) else FORMAT_VERSION_V1

    def to_bytes(self) -> bytes:
        out = io.BytesIO()
        self.write_to(out)
        return out.getvalue()

    def write_to(self, f: BinaryIO) -> None:
        hb = json.dumps(self.header(), separators=(",", ":")).encode("utf-8")
        f.write(MAGIC)
        f.write(struct.pack("<H", self.version()))
        f.write(struct.pack("<I", len(hb)))
        f.write(hb)
        f.write(self.data.getvalue())

    def write(self, path) -> str:
        with open(path, "wb") as f:
            self.write_to(f)
        return str(path)


def write_container(path, header: dict, data: bytes, format_version: int = FORMAT_VERSION_V1) -> None:
    """Reference-signature writer (bigsmall/container.py:59-82)."""
    if format_version not in SUPPORTED_VERSIONS:
        raise ValueError(f"Unsupported BigSmall format version {format_version!r}")
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<H", format_version))
        f.write(struct.pack("<I", len(hb)))
        f.write(hb)
        f.write(data)


def tensor_raw_bytes(t: dict) -> int:
    return n_elements(t["shape"]) * DTYPE_BYTES.get(t["dtype"], 1)


def info(path) -> dict[str, Any]:
    """Summary of a container without decoding (subset of bigsmall/container.py:170-268)."""
    p = Path(path)
    header, data_offset = read_header(p)
    total_raw = sum(tensor_raw_bytes(t) for t in header["tensors"])
    file_size = p.stat().st_size
    stats: dict[str, int] = dict(header.get("codec_stats") or {})
    if not stats:
        for t in header["tensors"]:
            stats[t["codec"]] = stats.get(t["codec"], 0) + 1
    return {"path": str(p), "file_size": file_size, "data_offset": data_offset,
            "tensor_count": header["tensor_count"], "estimated_raw_bytes": total_raw,
            "ratio_pct": file_size / total_raw * 100 if total_raw else 0.0, "codec_stats": stats,
            "format": header.get("format")}


def iter_blobs(header: dict, data: bytes | memoryview) -> Iterable[tuple[dict, memoryview]]:
    mv = memoryview(data)
    for t in header["tensors"]:
        yield t, mv[t["offset"]:t["offset"] + t["compressed_bytes"]]
