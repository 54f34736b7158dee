"""GPU backend of the reference's ``bigsmall.kernels`` module.

Same surface and probe state as BigSmall ``bigsmall/kernels/__init__.py:21-111``:
``_GPU_BACKEND`` (None before the first probe, ``""`` for no GPU backend,
``"cuda_c"`` otherwise), ``_GPU_DECODE_FN``, ``_probe_backend``, ``use_gpu``,
``backend_name`` (``"cpu"`` when there is no GPU backend) and
``decode_bf16_parallel``; ``BIGSMALL_FORCE_CPU`` disables the GPU backend as
there.  The backend is always this package's CUDA C library (the ``ac_cuda``
slot the reference probes first, ``:54-63``); there is no Triton backend, so
``BIGSMALL_FORCE_TRITON`` changes nothing.  Two deliberate differences: this
package has no CPU decoder, so decoding without a GPU backend raises instead of
running one, and a CUDA device whose library is missing or broken raises at the
probe instead of falling back (``:97-111`` swallows such errors into a
warning).
"""
from __future__ import annotations

import os
from typing import Optional

_GPU_BACKEND: Optional[str] = None   # None: not probed yet; "": no GPU backend; "cuda_c"
_GPU_DECODE_FN = None                # set by the probe


def _force_cpu() -> bool:
    return os.environ.get("BIGSMALL_FORCE_CPU", "").lower() in ("1", "true", "yes")


def _probe_backend() -> None:
    """Decide (once) whether the CUDA C backend is used."""
    global _GPU_BACKEND, _GPU_DECODE_FN
    if _GPU_BACKEND is not None:
        return
    if _force_cpu():
        _GPU_BACKEND = ""
        return
    import torch
    if not torch.cuda.is_available():
        _GPU_BACKEND = ""
        return
    from . import ac_cuda        # loads libbsgpu.so; raises if it is missing
    _GPU_DECODE_FN = ac_cuda.decode
    _GPU_BACKEND = "cuda_c"


def use_gpu() -> bool:
    """True if the CUDA C backend is available and will be used."""
    _probe_backend()
    return bool(_GPU_BACKEND)


def backend_name() -> str:
    _probe_backend()
    return _GPU_BACKEND or "cpu"


def decode_bf16_parallel(blob: bytes, extras: dict, n_weights: int) -> bytes:
    """Decode a ``bf16_parallel_v1`` blob to raw bf16 bytes on the GPU."""
    _probe_backend()
    if not _GPU_BACKEND or _GPU_DECODE_FN is None:
        raise RuntimeError(
            "bigsmall_b200 decodes on the GPU only and no GPU backend is in use "
            + ("(BIGSMALL_FORCE_CPU is set)" if _force_cpu() else "(no CUDA device)")
            + "; the reference's bigsmall.codecs.bf16_parallel.decode is the CPU decoder")
    return _GPU_DECODE_FN(blob, extras, n_weights)
