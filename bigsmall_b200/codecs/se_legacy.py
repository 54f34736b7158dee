"""Legacy serial BigSmall formats decoded on the device: ``bf16_se_single_kernel``
(BigSmall ``bigsmall/codecs/single_kernel.py:432-613``) and ``bf16_se_tans``
(``bigsmall/codecs/bf16_tans.py:121-167`` with ``numba_rans.py:168-217``).

Both hold one serial (sign,exp) rANS stream per tensor plus one rANS stream
per exponent bucket of mantissas.  The device decodes all of a tensor's
streams concurrently (one CTA each) and un-sorts on the device, so a tensor
takes the time of its (sign,exp) stream: bit-exact, latency-bound, and no
faster than one CPU core per tensor; a container's tensors decode in parallel.
There is no device encoder for these formats: blobs come from the reference.
Errors mirror the reference decoders' (count mismatch, truncation, corrupt
tables) as ``ValueError`` subclasses.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import gpu

CODECS = tuple(gpu.SE_CODECS)


def encode(raw: bytes, **_):
    raise NotImplementedError("legacy serial blobs are produced by the reference encoder; "
                              "bigsmall_b200 encodes bf16_exp_chunked_v1")


def decode_to_device(codec: str, blob: bytes, extras: dict, n_weights: int, device=None) -> torch.Tensor:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = torch.empty(max(n_weights, 1), dtype=torch.int16, device=dev)
    b = bytes(blob)
    d = torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).to(dev) if b else None
    gpu.decode_se_into(codec, b, d, out, n_weights)
    return out[:n_weights]


def decoder_for(codec: str):
    """The reference's ``decode(blob, extras, n_weights) -> bytes`` contract."""
    def decode(blob: bytes, extras: dict, n_weights: int) -> bytes:
        if n_weights == 0 or len(blob) == 0:
            return b""
        return decode_to_device(codec, blob, extras, n_weights).cpu().numpy().tobytes()
    decode.__name__ = f"decode_{codec}"
    return decode
