"""``bf16_exp_chunked_v1``: chunked exponent rANS/tANS/pair-rANS + raw sign|mantissa plane.

Host-bytes front-end of the device codec (the format is described in
``bigsmall_b200/csrc/common.cuh``).  ``decode`` uploads the blob, decodes on the
GPU and returns the bf16 bytes, so it can sit in the reference's codec
registry (``bigsmall/codec_registry.py:45-47``); device-resident callers use
:mod:`bigsmall_b200.gpu` / :mod:`bigsmall_b200.loader` and never touch host
bytes.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import gpu

CODEC = "bf16_exp_chunked_v1"


def _device(device=None) -> torch.device:
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device(device)


def encode(raw: bytes, coder: str = gpu.DEFAULT_CODER, prec: int = gpu.DEFAULT_PREC,
           chunk_elems: int = gpu.DEFAULT_CHUNK_ELEMS, device=None, groups: int = 1, **_) -> tuple[bytes, dict]:
    if len(raw) % 2 != 0:
        raise ValueError(f"BF16 byte length must be even, got {len(raw)}")
    if len(raw) == 0:
        return b"", gpu.xc_extras(chunk_elems, coder, prec, groups)
    dev = _device(device)
    x = torch.from_numpy(np.frombuffer(raw, dtype=np.int16).copy()).to(dev)
    blob = gpu.encode_xc(x, coder=coder, prec=prec, chunk_elems=chunk_elems, groups=groups)
    return blob.cpu().numpy().tobytes(), gpu.xc_extras(chunk_elems, coder, prec, groups)


def decode_to_device(blob, extras: dict, n_weights: int, device=None) -> torch.Tensor:
    """Decode to a device int16 tensor (bit pattern of the bf16 values)."""
    dev = _device(device)
    out = torch.empty(n_weights, dtype=torch.int16, device=dev)
    if n_weights == 0:
        return out
    if isinstance(blob, torch.Tensor):
        d = blob if blob.is_cuda else blob.to(dev)
    else:
        d = torch.from_numpy(np.frombuffer(bytes(blob), dtype=np.uint8).copy()).to(dev)
    if d.data_ptr() % 16:
        d = d.clone()
    ce = int((extras or {}).get("chunk_elems", gpu.DEFAULT_CHUNK_ELEMS))
    gpu.decode_xc_into(d, out, ce, coder=(extras or {}).get("coder"), groups=gpu.extras_groups(extras))
    return out


def decode(blob: bytes, extras: dict, n_weights: int) -> bytes:
    if n_weights == 0 or len(blob) == 0:
        return b""
    return decode_to_device(blob, extras, n_weights).cpu().numpy().tobytes()
