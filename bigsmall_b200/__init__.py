"""bigsmall_b200 -- B200-native (sm_100a) engine for BigSmall's bf16 decode path.

Decodes a ``.bs`` container's entropy-coded bf16 tensors straight into HBM
with hand-written CUDA kernels behind a C ABI (``include/bsgpu.h``,
``bigsmall_b200/libbsgpu.so``), and exposes them behind the reference's own
Python API shape (``decompress``/``load``/``_decode_blob``, the
``codec_registry``, ``StreamingLoader``, ``BigSmallStreamingModel``,
``CompressedKVCache`` and the ``kernels.ac_cuda`` backend slot).

Formats decoded on the device:
  * ``bf16_exp_chunked_v1`` -- this project's chunked exponent format (rANS,
    tANS or rANS over exponent pairs) with a raw sign|mantissa byte plane
    (the throughput format; device encoder included);
  * ``bf16_parallel_v1`` -- the reference's GPU-oriented rANS format
    (BigSmall ``bigsmall/codecs/bf16_parallel.py``), bit-exact;
  * ``bf16_se_single_kernel`` / ``bf16_se_tans`` -- the reference's serial
    formats, bit-exact (one serial stream per tensor).

Several GPUs: ``sharding`` cuts a container into per-rank chunk spans (decode
needs no communication) and ``replicate`` materialises the whole model on
every rank afterwards when wanted (NCCL point-to-point).

Top-level names follow BigSmall ``bigsmall/__init__.py`` for the decode path
(``decompress``, ``load``, ``verify``, ``info``, ``StreamingLoader``,
``BigSmallStreamingModel``) and are imported on first use, so importing the
package needs neither torch nor a GPU.
"""
from __future__ import annotations

__version__ = "0.1.0"

from .exceptions import BigSmallVersionError, BsCorruptError, BsGpuError  # noqa: F401

_LAZY = {
    "decompress": ("decoder", "decompress"),
    "load": ("decoder", "load"),
    "verify": ("decoder", "verify"),
    "compress_tensors": ("decoder", "compress_tensors"),
    "info": ("container", "info"),
    "StreamingLoader": ("streaming", "StreamingLoader"),
    "BigSmallStreamingModel": ("streaming_inference", "BigSmallStreamingModel"),
    "CompressedKVCache": ("kv_cache_manager", "CompressedKVCache"),
}

__all__ = ["BigSmallVersionError", "BsCorruptError", "BsGpuError", *_LAZY]


def __getattr__(name):
    if name in _LAZY:
        import importlib
        mod, attr = _LAZY[name]
        return getattr(importlib.import_module(f".{mod}", __name__), attr)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
