"""bigsmall_b200 -- B200-native (sm_100a) engine for BigSmall's bf16 decode path.

Decodes a ``.bs`` container's entropy-coded bf16 tensors straight into HBM
with hand-written CUDA kernels behind a C ABI (``include/bsgpu.h``,
``bigsmall_b200/libbsgpu.so``), and exposes them behind the reference's own
Python API shape (``decompress``/``load``/``_decode_blob``, the
``codec_registry``, ``StreamingLoader``, ``BigSmallStreamingModel``,
``CompressedKVCache`` and the ``kernels.ac_cuda`` backend slot).

Formats decoded on the device:
  * ``bf16_parallel_v1`` -- the reference's GPU-oriented rANS format
    (BigSmall ``bigsmall/codecs/bf16_parallel.py``), bit-exact;
  * ``bf16_exp_chunked_v1`` -- this project's chunked exponent rANS/tANS
    format with a raw sign|mantissa byte plane (the throughput format).
"""
from __future__ import annotations

__version__ = "0.1.0"

from .exceptions import BigSmallVersionError, BsCorruptError, BsGpuError  # noqa: F401
