"""KV-cache compression on the device.

Same blob framing as BigSmall ``bigsmall/codecs/kv_cache.py:51-60``::

    [u8 version][u8 ndim_k][i32 shape_k ...][u32 k_len][k blob]
                [u8 ndim_v][i32 shape_v ...][u32 v_len][v blob]

with a new version 3 whose blobs are bf16_exp_chunked_v1 (encoded and decoded
on the GPU).  Versions 1 and 2 hold constriction bitstreams (bf16_se_ac /
bf16_se_rans, ``kv_cache.py:92-95``); this package does not decode them.

The reference moves K/V to the host before encoding (``kv_cache.py:24-29``) and
back after decoding (``:32-38``); :func:`encode_kv` / :func:`decode_kv` keep
both sides in HBM, and the byte-level functions exist for drop-in use.
"""
from __future__ import annotations

import struct
from typing import Optional

import numpy as np
import torch

from . import gpu

KV_VERSION = 3
KV_CHUNK_ELEMS = gpu.DEFAULT_CHUNK_ELEMS


def _check_bf16(t: torch.Tensor, what: str) -> None:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{what} must be BF16 tensors, got {t.dtype}")


class KVEncoder:
    """Reusable device encoder for K/V tensors (grows its buffers on demand).

    A layer's K and V are encoded concurrently by two encoders (each with its
    own workspace and output buffer), the second on a side stream: one
    tensor's per-chunk encode kernel leaves most of the GPU idle (one warp per
    chunk), so two in flight keep more SMs busy."""

    def __init__(self, device=None, chunk_elems: int = KV_CHUNK_ELEMS, coder: str = gpu.DEFAULT_CODER):
        self.device = torch.device("cuda", device if isinstance(device, int) else
                                   (torch.device(device).index if device is not None else torch.cuda.current_device()))
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.chunk_elems = chunk_elems
        self.coder = coder
        self._encs: list = [None, None]
        self._side: Optional[torch.cuda.Stream] = None

    def encoder(self, n: int, k: int = 0) -> gpu.XcEncoder:
        e = self._encs[k]
        if e is None or e.max_elems < n:
            e = self._encs[k] = gpu.XcEncoder(max(n, 1), self.chunk_elems, self.coder, device=self.device.index)
        return e

    def _flat(self, t: torch.Tensor) -> torch.Tensor:
        x = t.detach().contiguous().reshape(-1)
        return x if x.device == self.device else x.to(self.device)

    def encode(self, t: torch.Tensor) -> torch.Tensor:
        """Right-sized device blob of one tensor (synchronises to read the size)."""
        x = self._flat(t)
        return self.encoder(x.numel()).encode(x)

    def encode_pair(self, keys: torch.Tensor, values: torch.Tensor):
        """Right-sized device blobs of K and V, encoded concurrently on the
        current stream and a side stream (one synchronisation for both sizes)."""
        xk, xv = self._flat(keys), self._flat(values)
        ek, ev = self.encoder(xk.numel(), 0), self.encoder(xv.numel(), 1)
        main = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        self._side.wait_stream(main)
        ek.encode_async(xk, main)
        ev.encode_async(xv, self._side)
        main.wait_stream(self._side)
        xv.record_stream(self._side)
        nk, nv = (int(v) for v in torch.stack([ek.out_len[0], ev.out_len[0]]).tolist())
        return ek.out[:nk].clone(), ev.out[:nv].clone()


def encode_kv(keys: torch.Tensor, values: torch.Tensor, enc: Optional[KVEncoder] = None):
    """(k_blob, v_blob) device uint8 tensors for one layer's K and V."""
    _check_bf16(keys, "keys")
    _check_bf16(values, "values")
    enc = enc or KVEncoder(keys.device if keys.is_cuda else None)
    return enc.encode_pair(keys, values)


def decode_kv(k_blob: torch.Tensor, v_blob: torch.Tensor, k_shape, v_shape, device=None,
              chunk_elems: int = KV_CHUNK_ELEMS, out: Optional[tuple] = None, coder=None):
    """Decode both blobs (device) with one plan; returns (keys, values) bf16."""
    dev = k_blob.device if device is None else torch.device(device)
    if out is None:
        k = torch.empty(tuple(k_shape), dtype=torch.bfloat16, device=dev)
        v = torch.empty(tuple(v_shape), dtype=torch.bfloat16, device=dev)
    else:
        k, v = out
    entries = [(b, o.view(torch.int16).reshape(-1), chunk_elems) for b, o in ((k_blob, k), (v_blob, v)) if o.numel()]
    if entries:
        with gpu.XcPlan(entries, device=dev.index, coders=coder) as p:
            p.run()
    return k, v


def compress_kv_entry(keys: torch.Tensor, values: torch.Tensor) -> bytes:
    """Version-3 KV blob (bytes) of one layer; encoded on the GPU."""
    kb, vb = encode_kv(keys.cuda() if not keys.is_cuda else keys, values.cuda() if not values.is_cuda else values)
    out = bytearray()
    out += struct.pack("<B", KV_VERSION)
    for shape, blob in ((keys.shape, kb), (values.shape, vb)):
        out += struct.pack("<B", len(shape))
        for s in shape:
            out += struct.pack("<i", int(s))
        b = blob.cpu().numpy().tobytes()
        out += struct.pack("<I", len(b))
        out += b
    return bytes(out)


def _parse(data: bytes):
    pos = 0
    version = data[pos]
    pos += 1
    if version != KV_VERSION:
        if version in (1, 2):
            raise ValueError(f"KV cache codec version {version} holds constriction bitstreams "
                             "(bf16_se_ac / bf16_se_rans); bigsmall_b200 decodes version 3")
        raise ValueError(f"Unknown KV cache codec version {version}")
    parts = []
    for _ in range(2):
        ndim = data[pos]
        pos += 1
        shape = [struct.unpack_from("<i", data, pos + 4 * i)[0] for i in range(ndim)]
        pos += 4 * ndim
        blen, = struct.unpack_from("<I", data, pos)
        pos += 4
        parts.append((shape, data[pos:pos + blen]))
        pos += blen
    return parts


def decompress_kv_entry(data: bytes, device: str = "cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of :func:`compress_kv_entry`; tensors are decoded on ``device``."""
    (ks, kb), (vs, vb) = _parse(data)
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("KV blobs are decoded on a CUDA device")
    def up(b):
        return torch.from_numpy(np.frombuffer(bytes(b), dtype=np.uint8).copy()).to(dev)
    return decode_kv(up(kb), up(vb), ks, vs, device=dev)
