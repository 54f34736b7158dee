"""The ``bigsmall.kernels.ac_cuda`` backend module the reference probes for
(BigSmall ``bigsmall/kernels/__init__.py:54-63``; the module does not exist in
the reference).

Contract of the slot: ``decode(blob, extras, n_weights) -> bytes`` for
``bf16_parallel_v1`` blobs, bit-identical to the CPU decoder
(``bigsmall/codecs/bf16_parallel.py:262-352``), with its errors (``ValueError``
on bad magic, precision or count).  ``decode_to_device`` is the same decode
leaving the values in HBM (an int16 view of the bf16 words), for callers that
would otherwise copy the bytes back to the device (``bigsmall/decoder.py:301-310``
decodes to host memory and then moves the tensor).
"""
from __future__ import annotations

from ..codecs import bf16_parallel as _par


def decode(blob: bytes, extras: dict, n_weights: int) -> bytes:
    return _par.decode(blob, extras, n_weights)


def decode_to_device(blob: bytes, extras: dict, n_weights: int, device=None):
    return _par.decode_to_device(blob, extras, n_weights, device)
