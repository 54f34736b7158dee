"""GPU backend of the reference's ``bigsmall.kernels`` module.

Same surface as BigSmall ``bigsmall/kernels/__init__.py:36-111``
(``use_gpu``, ``backend_name``, ``decode_bf16_parallel``), but the backend is
always this package's CUDA C extension (the ``ac_cuda`` slot the reference
probes first, ``:56-64``) and there is no silent CPU fallback: a device error
raises instead of being swallowed into a warning (``:97-111``).
"""
from __future__ import annotations

from . import ac_cuda


def use_gpu() -> bool:
    import torch
    return torch.cuda.is_available()


def backend_name() -> str:
    return "cuda_c" if use_gpu() else "unavailable"


def decode_bf16_parallel(blob: bytes, extras: dict, n_weights: int) -> bytes:
    return ac_cuda.decode(blob, extras, n_weights)
