"""``bf16_parallel_v1`` (the reference's GPU-oriented format) decoded on the device.

Bit-exact with BigSmall ``bigsmall/codecs/bf16_parallel.py:262-352``; errors
mirror it (bad magic / precision mismatch / weight count mismatch raise
``ValueError``).  There is no device encoder for this legacy format: blobs
come from the reference's CPU encoder.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import gpu

CODEC = "bf16_parallel_v1"


def encode(raw: bytes, **_):
    raise NotImplementedError("bf16_parallel_v1 blobs are produced by the reference encoder; "
                              "bigsmall_b200 encodes bf16_exp_chunked_v1")


def decode_to_device(blob: bytes, extras: dict, n_weights: int, device=None) -> torch.Tensor:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = torch.empty(max(n_weights, 1), dtype=torch.int16, device=dev)
    b = bytes(blob)
    d = torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).to(dev) if b else None
    gpu.decode_par_into(b, d, out, n_weights)
    return out[:n_weights]


def decode(blob: bytes, extras: dict, n_weights: int) -> bytes:
    if n_weights == 0 or len(blob) == 0:
        return b""
    return decode_to_device(blob, extras, n_weights).cpu().numpy().tobytes()
