"""The ``bigsmall.kernels.ac_cuda`` backend module the reference probes for
(BigSmall ``bigsmall/kernels/__init__.py:56-64``; the module does not exist in
the reference).  Contract: ``decode(blob, extras, n_weights) -> bytes`` for
``bf16_parallel_v1`` blobs, bit-identical to the CPU decoder."""
from __future__ import annotations

from ..codecs import bf16_parallel as _par


def decode(blob: bytes, extras: dict, n_weights: int) -> bytes:
    return _par.decode(blob, extras, n_weights)
